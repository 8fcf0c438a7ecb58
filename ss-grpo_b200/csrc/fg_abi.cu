// fg_abi.cu -- housekeeping entry points of the C ABI: version, status
// strings, the per-device error word and the bounded-wait check.
#include <cstdio>

#include "fg_common.cuh"

// First FG_* status a kernel recorded on this device (0 = none).
__device__ int32_t g_fg_error_word = 0;

namespace fg {

// Cache row of call row b under a row map (fg_kv_layer.rows): -1 (and
// FG_EINVAL recorded) when the mapped row lies outside the cache.
__device__ __forceinline__ int32_t cache_row(const int32_t* rows, int32_t batch, int32_t b) {
    if (rows == nullptr) return b;
    const int32_t r = rows[b];
    if (r < 0 || r >= batch) {
        atomicCAS(&g_fg_error_word, 0, FG_EINVAL);
        return -1;
    }
    return r;
}

static thread_local int32_t t_last_cuda_error = 0;

void set_cuda_error(cudaError_t e) { t_last_cuda_error = (int32_t)e; }

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for *flag != 0 for at most timeout_ns; reports FG_OK / FG_ETIMEOUT.
__global__ void wait_flag_kernel(const int32_t* flag, int64_t timeout_ns, int32_t* status_out) {
    if (threadIdx.x != 0) return;
    const uint64_t start = global_ns();
    int32_t status = FG_ETIMEOUT;
    for (uint32_t it = 0; it < (1u << 30); ++it) {
        if (*(volatile const int32_t*)flag != 0) {
            status = FG_OK;
            break;
        }
        if ((int64_t)(global_ns() - start) > timeout_ns) break;
        __nanosleep(1000);
    }
    *status_out = status;
    if (status != FG_OK) atomicCAS(&g_fg_error_word, 0, status);
}

}  // namespace fg

extern "C" const char* fg_version(void) { return "fg_b200 0.1.0 (sm_100a)"; }

extern "C" const char* fg_status_string(fg_status s) {
    switch (s) {
        case FG_OK: return "ok";
        case FG_EINVAL: return "invalid argument";
        case FG_ECAPACITY: return "capacity exceeded";
        case FG_ETIMEOUT: return "device wait timed out";
        case FG_ECUDA: return "CUDA error";
        case FG_EUNSUPPORTED: return "unsupported configuration";
        default: return "unknown status";
    }
}

extern "C" int32_t fg_last_cuda_error(void) { return fg::t_last_cuda_error; }

extern "C" fg_status fg_read_device_error(int32_t* host_out, int32_t clear) {
    if (!host_out) return FG_EINVAL;
    cudaError_t e = cudaMemcpyFromSymbol(host_out, g_fg_error_word, sizeof(int32_t));
    if (e != cudaSuccess) {
        fg::set_cuda_error(e);
        return FG_ECUDA;
    }
    if (clear) {
        const int32_t zero = 0;
        e = cudaMemcpyToSymbol(g_fg_error_word, &zero, sizeof(int32_t));
        if (e != cudaSuccess) {
            fg::set_cuda_error(e);
            return FG_ECUDA;
        }
    }
    return FG_OK;
}

extern "C" fg_status fg_wait_flag(const int32_t* flag, int64_t timeout_ns, int32_t* status_out, void* stream) {
    if (!flag || !status_out || timeout_ns < 0) return FG_EINVAL;
    fg::wait_flag_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(flag, timeout_ns, status_out);
    return fg::launch_status();
}

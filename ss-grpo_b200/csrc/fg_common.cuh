// fg_common.cuh -- shared device helpers for the sm_100a tree-verify kernels.
//
// Holds the status plumbing of the C ABI, element loads for the three
// logits/activation dtypes, Philox4x32-10, and the sampler exp.  The sampler
// arithmetic follows the "fg-icdf-v1" specification written out in
// include/fg_b200.h; every floating-point step uses an explicit round-to-
// nearest intrinsic so the compiler cannot contract or reorder it, which is
// what makes the GPU draw the same token as the CPU checker.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fg_b200.h"

#define FG_SAMPLE_LANES 512

namespace fg {

// Records the last CUDA error seen by an entry point (per process).
void set_cuda_error(cudaError_t e);

inline int32_t launch_status() {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return FG_ECUDA;
    }
    return FG_OK;
}

// Launch as a programmatic dependent of the preceding kernel on the stream:
// the grid may start while that kernel finishes, so the kernel itself must
// execute griddepcontrol.wait before it reads anything the preceding kernels
// wrote (every kernel launched this way does so first, then lets its own
// dependents launch).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// The grid dependency of a kernel launched with launch_pdl: wait for the
// preceding kernel, then let the next one launch.
__device__ __forceinline__ void pdl_wait_then_release() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float load_elem(const void* p, int32_t dtype, int64_t i) {
    if (dtype == FG_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    if (dtype == FG_DTYPE_F16) return __half2float(static_cast<const __half*>(p)[i]);
    return static_cast<const float*>(p)[i];
}

// ------------------------------------------------------------------ Philox
// Philox4x32-10, Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3" (SC'11): two 32x32->64 multiplies per round with the
// published multipliers, Weyl-sequence key schedule, ten rounds.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        if (r > 0) {
            k.x += 0x9E3779B9u;
            k.y += 0xBB67AE85u;
        }
        const uint32_t lo0 = 0xD2511F53u * c.x;
        const uint32_t hi0 = __umulhi(0xD2511F53u, c.x);
        const uint32_t lo1 = 0xCD9E8D57u * c.z;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z);
        c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    }
    return c;
}

__device__ __forceinline__ float philox_uniform(uint64_t seed, uint32_t seq, uint32_t round_idx, uint32_t draw) {
    const uint4 o = philox4x32_10(make_uint4(seq, round_idx, draw, 0u),
                                  make_uint2((uint32_t)(seed & 0xffffffffu), (uint32_t)(seed >> 32)));
    return __fmul_rn((float)(o.x >> 8), 0x1p-24f);
}

// --------------------------------------------------------------- sampler exp
// Cody-Waite reduction x = n ln2 + r (ln2 split into a 16-significant-bit
// head and its fp32 tail so n * head is exact), degree-7 Taylor polynomial of
// e^r by fused Horner steps with coefficients fp32(1/k!), scale by 2^n via the
// exponent field.  Inputs below -86 (and NaN) give 0.
// n = rint(t), ties to even, without the conversion units: for |t| < 2^22,
// t + 1.5 * 2^23 lands where the float spacing is 1, so round-to-nearest-even
// leaves the integer nearest t (ties to the even one, 1.5 * 2^23 being even)
// in the low significand bits; subtracting the constant back is exact.  The
// callers pass x - max <= 0, so t is in [-125, 0].
__device__ __forceinline__ float fg_exp(float x) {
    if (!(x >= -86.0f)) return 0.0f;
    const float t = __fmul_rn(x, 1.44269502162933349609375f);
    const float shifted = __fadd_rn(t, 12582912.0f);  // 1.5 * 2^23, bits 0x4B400000
    const float nf = __fsub_rn(shifted, 12582912.0f);
    const int n = __float_as_int(shifted) - 0x4B400000;
    float r = __fmaf_rn(-nf, 0.693145751953125f, x);
    r = __fmaf_rn(-nf, 1.42860676533018704503775e-06f, r);
    float p = 1.98412701138295233249664e-04f;
    p = __fmaf_rn(p, r, 1.38888892251998186111450e-03f);
    p = __fmaf_rn(p, r, 8.33333376795053482055664e-03f);
    p = __fmaf_rn(p, r, 4.16666679084300994873047e-02f);
    p = __fmaf_rn(p, r, 1.66666671633720397949219e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    return __fmul_rn(p, __int_as_float((n + 127) << 23));
}

__host__ __device__ __forceinline__ int32_t sample_chunk_len(int32_t V) {
    int32_t c = (V + FG_SAMPLE_LANES - 1) / FG_SAMPLE_LANES;
    return (c + 7) & ~7;
}

__device__ __forceinline__ float scaled_logit(const void* row, int32_t dtype, int32_t i, float temperature) {
    float v = load_elem(row, dtype, i);
    if (temperature > 0.0f) v = __fdiv_rn(v, temperature);
    return v;
}

// --------------------------------------------------------- cluster helpers
// Rank of this CTA in its thread-block cluster.
__device__ __forceinline__ uint32_t cl_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Every thread of every CTA of the cluster arrives and waits; shared-memory
// writes before it are visible to the cluster's loads after it.
__device__ __forceinline__ void cl_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of CTA `rank`'s copy of the shared variable at
// `p` (distributed shared memory).
__device__ __forceinline__ uint32_t cl_addr(const void* p, uint32_t rank) {
    uint32_t local = static_cast<uint32_t>(__cvta_generic_to_shared(p)), remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
    return remote;
}

// ---------------------------------------------------------- block helpers
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace fg

// fg_sampler.cuh -- block-wide fg-icdf-v1 draw and greedy argmax.
//
// One CTA of FG_SAMPLE_LANES threads draws one token from one logits row.
// Thread t owns vocabulary chunk t (C = roundup8(ceil(V / 512)) contiguous
// entries); the chunk totals are prefix-summed sequentially by thread 0 so
// the cumulative values are exactly those of the CPU checker.
#pragma once

#include "fg_common.cuh"

namespace fg {

struct SampleSmem {
    float P[FG_SAMPLE_LANES + 1];
    float red[FG_SAMPLE_LANES / 32];
    int32_t redi[FG_SAMPLE_LANES / 32];
    int32_t result;
};

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ float scaled_t(const T* row, int32_t i, float temperature) {
    float v = to_f<T>(row[i]);
    if (temperature > 0.0f) v = __fdiv_rn(v, temperature);
    return v;
}

// First index of the maximum (torch.argmax); ties -> lower index.
template <typename T>
__device__ int32_t block_argmax(const T* row, int32_t V, SampleSmem& sm) {
    const int tid = threadIdx.x;
    float bv = -INFINITY;
    int32_t bi = 0x7fffffff;
    for (int32_t i = tid; i < V; i += FG_SAMPLE_LANES) {
        const float v = to_f<T>(row[i]);
        if (v > bv) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if ((tid & 31) == 0) {
        sm.red[tid >> 5] = bv;
        sm.redi[tid >> 5] = bi;
    }
    __syncthreads();
    if (tid == 0) {
        float v = sm.red[0];
        int32_t i = sm.redi[0];
        for (int w = 1; w < FG_SAMPLE_LANES / 32; ++w)
            if (sm.red[w] > v || (sm.red[w] == v && sm.redi[w] < i)) {
                v = sm.red[w];
                i = sm.redi[w];
            }
        sm.result = (i == 0x7fffffff) ? 0 : i;
    }
    __syncthreads();
    const int32_t r = sm.result;
    __syncthreads();
    return r;
}

// fg-icdf-v1 draw; returns -1 only when every entry is NaN or -inf.
template <typename T>
__device__ int32_t block_sample(const T* row, int32_t V, float temperature, bool do_sample, float u, SampleSmem& sm) {
    if (!do_sample || temperature == 0.0f) return block_argmax<T>(row, V, sm);
    const int tid = threadIdx.x;
    // pass 1: row maximum (order independent, coalesced)
    float m = -INFINITY;
    for (int32_t i = tid; i < V; i += FG_SAMPLE_LANES) m = fmaxf(m, scaled_t<T>(row, i, temperature));
    m = warp_max(m);
    if ((tid & 31) == 0) sm.red[tid >> 5] = m;
    __syncthreads();
    if (tid < 32) {
        float v = tid < FG_SAMPLE_LANES / 32 ? sm.red[tid] : -INFINITY;
        v = warp_max(v);
        if (tid == 0) sm.red[0] = v;
    }
    __syncthreads();
    m = sm.red[0];
    // pass 2: left-to-right sum of this thread's chunk
    const int32_t C = sample_chunk_len(V);
    const int32_t lo = tid * C;
    const int32_t hi = min(lo + C, V);
    float c = 0.0f;
    for (int32_t i = lo; i < hi; ++i) c = __fadd_rn(c, fg_exp(__fsub_rn(scaled_t<T>(row, i, temperature), m)));
    sm.P[tid + 1] = c;
    if (tid == 0) sm.result = -1;
    __syncthreads();
    if (tid == 0) {
        float P = 0.0f;
        sm.P[0] = 0.0f;
        for (int t = 0; t < FG_SAMPLE_LANES; ++t) {
            P = __fadd_rn(P, sm.P[t + 1]);
            sm.P[t + 1] = P;
        }
    }
    __syncthreads();
    const float target = __fmul_rn(u, sm.P[FG_SAMPLE_LANES]);
    const float P0 = sm.P[tid];
    if (P0 <= target && target < sm.P[tid + 1]) {
        float cc = 0.0f;
        for (int32_t i = lo; i < hi; ++i) {
            cc = __fadd_rn(cc, fg_exp(__fsub_rn(scaled_t<T>(row, i, temperature), m)));
            if (__fadd_rn(P0, cc) > target) {
                sm.result = i;
                break;
            }
        }
    }
    __syncthreads();
    const int32_t r = sm.result;
    __syncthreads();
    return r;
}

}  // namespace fg

// fg_sampler.cuh -- block-wide fg-icdf-v1 draw and greedy argmax.
//
// One CTA of FG_SAMPLE_LANES threads draws one token from one logits row.
// Thread t owns vocabulary chunk t (C = roundup8(ceil(V / 512)) contiguous
// entries); the chunk totals are prefix-summed sequentially by thread 0 so
// the cumulative values are exactly those of the CPU checker.  Rows that
// allow it are read with 16-byte vectors, several in flight per thread; the
// order of every floating-point addition stays the specified one.
#pragma once

#include "fg_common.cuh"
#include "fg_vec.cuh"

namespace fg {

// Chunks up to this length are searched by a warp (exponentials in
// parallel, the running sum by one lane); longer ones by their own thread.
constexpr int kFindWarpMax = 1024;

struct SampleSmem {
    float P[FG_SAMPLE_LANES + 1];
    float e[kFindWarpMax];  // the searched chunk's e_i
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

// x / T (IEEE division) for T > 0.  Division by 1 is exact, so T == 1 skips
// it and gives the same value.
__device__ __forceinline__ float scale_t(float v, float temperature) {
    return temperature > 0.0f && temperature != 1.0f ? __fdiv_rn(v, temperature) : v;
}

// Block-wide (max value, lowest index) reduction; returns the index.
__device__ __forceinline__ int32_t block_best(float bv, int32_t bi, SampleSmem& sm) {
    const int tid = threadIdx.x;
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
        sm.red[0] = v;
    }
    __syncthreads();
    const int32_t r = sm.result;
    return r;
}

// Row maximum (raw values) and its first index.
template <typename T>
__device__ __forceinline__ void row_max(const T* row, int32_t V, float& bv, int32_t& bi) {
    bv = -INFINITY;
    bi = 0x7fffffff;
    const int tid = threadIdx.x;
    if (row_vectorizable<T>(row, V)) {
        constexpr int NV = Vec<T>::N;
        const int32_t nvec = V / NV;
        for (int32_t v0 = tid; v0 < nvec; v0 += 4 * FG_SAMPLE_LANES) {
            uint4 u[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int32_t v = v0 + k * FG_SAMPLE_LANES;
                u[k] = v < nvec ? ldg16(row + (int64_t)v * NV) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int32_t v = v0 + k * FG_SAMPLE_LANES;
                if (v >= nvec) break;
                float f[NV];
                unpack<T>(u[k], f);
#pragma unroll
                for (int e = 0; e < NV; ++e)
                    if (f[e] > bv) {
                        bv = f[e];
                        bi = v * NV + e;
                    }
            }
        }
    } else {
        for (int32_t i = tid; i < V; i += FG_SAMPLE_LANES) {
            const float x = to_f<T>(row[i]);
            if (x > bv) {
                bv = x;
                bi = i;
            }
        }
    }
}

// Left-to-right fp32 sum of e_i over [lo, hi).  With `target` >= 0 it
// instead returns the first i where base + running sum > target (or -1).
template <typename T, bool kFind>
__device__ __forceinline__ float chunk_scan(const T* row, int32_t lo, int32_t hi, float m, float temperature,
                                            bool vec, float base, float target, int32_t* found) {
    float c = 0.0f;
    if (vec) {
        constexpr int NV = Vec<T>::N;
        constexpr int NB = 4;
        for (int32_t i0 = lo; i0 < hi; i0 += NB * NV) {
            uint4 u[NB];
#pragma unroll
            for (int k = 0; k < NB; ++k)
                u[k] = (i0 + k * NV < hi) ? ldg16(row + i0 + k * NV) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int k = 0; k < NB; ++k) {
                if (i0 + k * NV >= hi) break;
                float f[NV];
                unpack<T>(u[k], f);
#pragma unroll
                for (int e = 0; e < NV; ++e) {
                    c = __fadd_rn(c, fg_exp(__fsub_rn(scale_t(f[e], temperature), m)));
                    if (kFind && __fadd_rn(base, c) > target) {
                        *found = i0 + k * NV + e;
                        return c;
                    }
                }
            }
        }
    } else {
        for (int32_t i = lo; i < hi; ++i) {
            c = __fadd_rn(c, fg_exp(__fsub_rn(scale_t(to_f<T>(row[i]), temperature), m)));
            if (kFind && __fadd_rn(base, c) > target) {
                *found = i;
                return c;
            }
        }
    }
    return c;
}

// First index of the maximum (torch.argmax); ties -> lower index.
template <typename T>
__device__ int32_t block_argmax(const T* row, int32_t V, SampleSmem& sm) {
    float bv;
    int32_t bi;
    row_max<T>(row, V, bv, bi);
    const int32_t r = block_best(bv, bi, sm);
    __syncthreads();
    return r;
}

// fg-icdf-v1 draw; returns -1 only when every entry is NaN or -inf.
template <typename T>
__device__ int32_t block_sample(const T* row, int32_t V, float temperature, bool do_sample, float u, SampleSmem& sm) {
    if (!do_sample || temperature == 0.0f) return block_argmax<T>(row, V, sm);
    const int tid = threadIdx.x;
    const int32_t C = sample_chunk_len(V);
    const int32_t lo = min(tid * C, V);
    const int32_t hi = min(lo + C, V);
    // pass 1: maximum of the scaled logits.  x -> x / T is monotone for T > 0,
    // so the maximum of the raw values, divided once, is that maximum.
    float bv;
    int32_t bi;
    row_max<T>(row, V, bv, bi);
    block_best(bv, bi, sm);
    const float m = scale_t(sm.red[0], temperature);
    __syncthreads();
    // pass 2: left-to-right sum of this thread's chunk
    const bool vec = row_vectorizable<T>(row, V);
    const float c = chunk_scan<T, false>(row, lo, hi, m, temperature, vec, 0.0f, 0.0f, nullptr);
    sm.P[tid + 1] = c;
    if (tid == 0) sm.result = -1;
    __syncthreads();
    if (tid == 0) {
        // the specified sequential sum, its loads batched ahead of the adds
        float P = 0.0f;
        sm.P[0] = 0.0f;
        for (int t0 = 0; t0 < FG_SAMPLE_LANES; t0 += 16) {
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = sm.P[t0 + j + 1];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                P = __fadd_rn(P, v[j]);
                sm.P[t0 + j + 1] = P;
            }
        }
    }
    __syncthreads();
    const float target = __fmul_rn(u, sm.P[FG_SAMPLE_LANES]);
    const float P0 = sm.P[tid];
    const bool mine = P0 <= target && target < sm.P[tid + 1];
    if (C > kFindWarpMax) {
        if (mine) {
            int32_t found = -1;
            chunk_scan<T, true>(row, lo, hi, m, temperature, vec, P0, target, &found);
            sm.result = found;
        }
    } else {
        // the chunk holding the target: its e_i computed by warp 0, then the
        // same left-to-right running sum by lane 0
        if (mine) sm.redi[0] = tid;
        if (tid == 0 && !(sm.P[0] <= target && target < sm.P[FG_SAMPLE_LANES])) sm.redi[0] = -1;
        __syncthreads();
        const int32_t t = sm.redi[0];
        if (tid < 32 && t >= 0) {
            const int32_t lo_t = min(t * C, V), hi_t = min(lo_t + C, V);
            for (int32_t i = lo_t + tid; i < hi_t; i += 32)
                sm.e[i - lo_t] = fg_exp(__fsub_rn(scale_t(to_f<T>(row[i]), temperature), m));
            __syncwarp();
            if (tid == 0) {
                const float base = sm.P[t];
                float c = 0.0f;
                int32_t found = -1;
                for (int32_t i = 0; i < hi_t - lo_t; ++i) {
                    c = __fadd_rn(c, sm.e[i]);
                    if (__fadd_rn(base, c) > target) {
                        found = lo_t + i;
                        break;
                    }
                }
                sm.result = found;
            }
        }
    }
    __syncthreads();
    const int32_t r = sm.result;
    __syncthreads();
    return r;
}

}  // namespace fg

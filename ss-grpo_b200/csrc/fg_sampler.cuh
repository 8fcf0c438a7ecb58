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
    alignas(16) float e[kFindWarpMax];  // the searched chunk's e_i
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

// The specified sequential prefix of the FG_SAMPLE_LANES chunk totals held
// in P[1 .. FG_SAMPLE_LANES], in place (P[0] = 0, P[t + 1] = P[t] + total t,
// left to right in fp32), by one thread: each batch of 8 totals is loaded
// while the previous batch is added.
__device__ __forceinline__ void sequential_prefix(float* P) {
    constexpr int kB = 8;
    float acc = 0.0f;
    P[0] = 0.0f;
    float v[kB], w[kB];
#pragma unroll
    for (int j = 0; j < kB; ++j) v[j] = P[j + 1];
    for (int t0 = 0; t0 < FG_SAMPLE_LANES; t0 += kB) {
        if (t0 + kB < FG_SAMPLE_LANES) {
#pragma unroll
            for (int j = 0; j < kB; ++j) w[j] = P[t0 + kB + j + 1];
        }
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            acc = __fadd_rn(acc, v[j]);
            P[t0 + j + 1] = acc;
        }
#pragma unroll
        for (int j = 0; j < kB; ++j) v[j] = w[j];
    }
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
// One warp writes e_i = fg_exp(x_i / T - m) of entries [lo, hi) (at most
// kFindWarpMax) of a row to e[0, hi - lo): whole 16-byte vectors, every lane's
// loads issued before they are used, when the row allows it.
template <typename T>
__device__ __forceinline__ void warp_chunk_exps(const T* row, int32_t lo, int32_t hi, float m, float temperature,
                                                bool vec, float* e) {
    const int lane = threadIdx.x & 31;
    constexpr int NV = Vec<T>::N;
    constexpr int PER = (kFindWarpMax / NV + 31) / 32;
    if (vec && lo % NV == 0) {
        const int32_t nv = (hi - lo) / NV;  // hi - lo is a multiple of NV here
        uint4 q[PER];
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int32_t v = lane + 32 * j;
            q[j] = v < nv ? ldg16(row + lo + (int64_t)v * NV) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int32_t v = lane + 32 * j;
            if (v < nv) {
                float f[NV];
                unpack<T>(q[j], f);
#pragma unroll
                for (int k = 0; k < NV; ++k) e[v * NV + k] = fg_exp(__fsub_rn(scale_t(f[k], temperature), m));
            }
        }
    } else {
        for (int32_t i = lo + lane; i < hi; i += 32) e[i - lo] = fg_exp(__fsub_rn(scale_t(to_f<T>(row[i]), temperature), m));
    }
    __syncwarp();
}

// The first i in [0, n) where base + (e[0] + ... + e[i]) > target, the sum
// taken left to right in fp32 (one lane), or -1.  The values are read 16 at
// a time ahead of their additions; the additions and comparisons are the
// sequential ones, and none happens past the answer.
__device__ __forceinline__ int32_t scan_chunk(const float* e, int32_t n, float base, float target) {
    float c = 0.0f;
    for (int32_t i0 = 0; i0 < n; i0 += 16) {
        float4 q[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) q[j] = reinterpret_cast<const float4*>(e + i0)[j];
        const float* v = reinterpret_cast<const float*>(q);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (i0 + j >= n) return -1;
            c = __fadd_rn(c, v[j]);
            if (__fadd_rn(base, c) > target) return i0 + j;
        }
    }
    return -1;
}

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
        sequential_prefix(sm.P);
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
            warp_chunk_exps<T>(row, lo_t, hi_t, m, temperature, vec, sm.e);
            if (tid == 0) {
                const int32_t i = scan_chunk(sm.e, hi_t - lo_t, sm.P[t], target);
                sm.result = i < 0 ? -1 : lo_t + i;
            }
        }
    }
    __syncthreads();
    const int32_t r = sm.result;
    __syncthreads();
    return r;
}

// ------------------------------------------------- cluster-wide fg-icdf-v1
// The draw of block_sample with a row spread over a cluster of S CTAs of NT
// threads; CTA r owns chunks [r * 512 / S, (r + 1) * 512 / S).
//   pass 1  every CTA takes the maximum of its part of the row and stores it
//           into every CTA (distributed shared memory); the row maximum is
//           the same value block_sample finds (only the value enters the
//           draw, as x - m: a signed zero gives the same e_i either way).
//   pass 2  in groups of kClusterChunkGroup chunks, all NT threads compute
//           the group's e_i = fg_exp(x_i / T - m) into shared memory (each
//           e_i alone, so they run in parallel), then thread c adds chunk
//           c's e_i left to right -- the chunk total of block_sample, the
//           same additions in the same order -- and stores it into CTA 0.
//   find    CTA 0 forms the sequential prefix of the 512 totals, finds the
//           target chunk and searches it exactly as block_sample does, and
//           stores the token into every CTA.
// All distributed-shared-memory traffic is stores before a cluster barrier
// and local reads after it, so no CTA reads a peer's memory after the peer
// may have exited.
constexpr int kClusterChunkGroup = 32;

template <int S, int NT>
struct ClusterSampleSmem {
    float P[FG_SAMPLE_LANES + 1];  // chunk totals, then their prefix (CTA 0)
    alignas(16) float e[kFindWarpMax];  // the searched chunk's e_i (CTA 0)
    float mv[S];                   // every CTA's maximum
    float red[NT / 32];
    int32_t target_chunk;
    int32_t result;
};

// Floats of the e_i buffer (dynamic shared memory) for vocabulary V: one
// group of chunks, each row padded to a multiple of 4 floats plus 4 so the
// summing threads' 16-byte reads fall in distinct banks.
__host__ __device__ __forceinline__ int32_t cluster_ebuf_stride(int32_t V) { return sample_chunk_len(V) + 4; }
__host__ __device__ __forceinline__ int64_t cluster_ebuf_bytes(int32_t V) {
    return (int64_t)kClusterChunkGroup * cluster_ebuf_stride(V) * 4;
}

// st.shared::cluster of one value into CTA `rank`'s copy of the variable.
__device__ __forceinline__ void cl_st_f32(float* p, uint32_t rank, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cl_addr(p, rank)), "f"(v) : "memory");
}
__device__ __forceinline__ void cl_st_s32(int32_t* p, uint32_t rank, int32_t v) {
    asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(cl_addr(p, rank)), "r"(v) : "memory");
}

template <typename T, int S, int NT>
__device__ int32_t cluster_sample(const T* row, int32_t V, float temperature, float u, ClusterSampleSmem<S, NT>& cs,
                                  float* ebuf) {
    constexpr int CPC = FG_SAMPLE_LANES / S;  // chunks per CTA
    static_assert(CPC % kClusterChunkGroup == 0, "chunk groups tile a CTA's chunks");
    const int tid = threadIdx.x;
    const uint32_t rank = cl_rank();
    const int32_t C = sample_chunk_len(V);
    const bool vec = row_vectorizable<T>(row, V);
    constexpr int NV = Vec<T>::N;
    // pass 1: maximum of this CTA's part [rank * CPC * C, ...) of the row
    {
        const int32_t lo = min((int32_t)rank * CPC * C, V), hi = min(lo + CPC * C, V);
        float bv = -INFINITY;
        if (vec) {
            const int32_t nvec = (hi - lo) / NV;  // lo, hi: multiples of C (a multiple of 8) or V
            const T* base = row + lo;
            for (int32_t v0 = tid; v0 < nvec; v0 += 8 * NT) {
                uint4 q[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int32_t v = v0 + k * NT;
                    q[k] = v < nvec ? ldg16(base + (int64_t)v * NV) : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    if (v0 + k * NT >= nvec) break;
                    float f[NV];
                    unpack<T>(q[k], f);
#pragma unroll
                    for (int e = 0; e < NV; ++e) bv = fmaxf(bv, f[e]);
                }
            }
        } else {
            for (int32_t i = lo + tid; i < hi; i += NT) bv = fmaxf(bv, to_f<T>(row[i]));
        }
        bv = warp_max(bv);
        if ((tid & 31) == 0) cs.red[tid >> 5] = bv;
        __syncthreads();
        if (tid < S) {
            float m = cs.red[0];
#pragma unroll
            for (int w = 1; w < NT / 32; ++w) m = fmaxf(m, cs.red[w]);
            cl_st_f32(&cs.mv[rank], tid, m);
        }
    }
    cl_sync();  // (A) every CTA holds every CTA's maximum
    float mraw = cs.mv[0];
#pragma unroll
    for (int r = 1; r < S; ++r) mraw = fmaxf(mraw, cs.mv[r]);
    const float m = scale_t(mraw, temperature);
    // pass 2: e_i of a group of chunks in parallel, then each chunk's total
    const int32_t stride = cluster_ebuf_stride(V);
    for (int grp = 0; grp < CPC; grp += kClusterChunkGroup) {
        const int32_t c0 = (int32_t)rank * CPC + grp;  // first (global) chunk of the group
        if (vec) {
            // the group's vectors (chunk, vector) dealt round-robin; a batch
            // of kBatch loads is issued before any is used
            constexpr int kBatch = 6;
            const int32_t vpc = C / NV;  // vectors per chunk
            const int32_t items = kClusterChunkGroup * vpc;
            for (int32_t it0 = tid; it0 < items; it0 += kBatch * NT) {
                uint4 q[kBatch];
                int32_t at[kBatch];
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const int32_t it = it0 + j * NT;
                    const int32_t lc = it / vpc, v = it - lc * vpc;
                    const int32_t i0 = (c0 + lc) * C + v * NV;
                    at[j] = (it < items && i0 < V) ? lc * stride + v * NV : -1;
                    q[j] = at[j] >= 0 ? ldg16(row + i0) : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    if (at[j] < 0) continue;
                    float f[NV];
                    unpack<T>(q[j], f);
                    float* dst = ebuf + at[j];
#pragma unroll
                    for (int e = 0; e < NV; e += 4)
                        *reinterpret_cast<float4*>(dst + e) =
                            make_float4(fg_exp(__fsub_rn(scale_t(f[e], temperature), m)),
                                        fg_exp(__fsub_rn(scale_t(f[e + 1], temperature), m)),
                                        fg_exp(__fsub_rn(scale_t(f[e + 2], temperature), m)),
                                        fg_exp(__fsub_rn(scale_t(f[e + 3], temperature), m)));
                }
            }
        } else {
            for (int32_t it = tid; it < kClusterChunkGroup * C; it += NT) {
                const int32_t lc = it / C, o = it - lc * C;
                const int32_t i = (c0 + lc) * C + o;
                if (i < V) ebuf[lc * stride + o] = fg_exp(__fsub_rn(scale_t(to_f<T>(row[i]), temperature), m));
            }
        }
        __syncthreads();
        if (tid < kClusterChunkGroup) {
            const int32_t g = c0 + tid;
            const int32_t n = max(0, min(g * C + C, V) - g * C);  // entries of chunk g
            const float* src = ebuf + tid * stride;
            float c = 0.0f;
            int32_t i = 0;
            // 16 values loaded ahead of their 16 additions
            for (; i + 16 <= n; i += 16) {
                float4 q[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) q[j] = *reinterpret_cast<const float4*>(src + i + 4 * j);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    c = __fadd_rn(c, q[j].x);
                    c = __fadd_rn(c, q[j].y);
                    c = __fadd_rn(c, q[j].z);
                    c = __fadd_rn(c, q[j].w);
                }
            }
            for (; i < n; ++i) c = __fadd_rn(c, src[i]);
            cl_st_f32(&cs.P[g + 1], 0, c);
        }
        __syncthreads();  // the next group overwrites the buffer
    }
    cl_sync();  // (B) CTA 0 holds the 512 chunk totals
    if (rank == 0) {
        if (tid == 0) {
            sequential_prefix(cs.P);
            cs.target_chunk = -1;
        }
        __syncthreads();
        const float target = __fmul_rn(u, cs.P[FG_SAMPLE_LANES]);
        for (int t = tid; t < FG_SAMPLE_LANES; t += NT)
            if (cs.P[t] <= target && target < cs.P[t + 1]) cs.target_chunk = t;
        __syncthreads();
        const int32_t t = cs.target_chunk;
        if (tid < 32) {
            int32_t found = -1;
            if (t >= 0) {
                const int32_t lo_t = min(t * C, V), hi_t = min(lo_t + C, V);
                warp_chunk_exps<T>(row, lo_t, hi_t, m, temperature, vec, cs.e);
                if (tid == 0) {
                    const int32_t i = scan_chunk(cs.e, hi_t - lo_t, cs.P[t], target);
                    found = i < 0 ? -1 : lo_t + i;
                }
            }
            const int32_t tok = __shfl_sync(0xffffffffu, found, 0);
            if (tid < S) cl_st_s32(&cs.result, tid, tok);
        }
    }
    cl_sync();  // (C) every CTA holds the token
    return cs.result;
}

}  // namespace fg

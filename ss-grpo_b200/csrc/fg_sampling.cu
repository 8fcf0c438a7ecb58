// fg_sampling.cu -- Philox uniforms, root-token sampling, row top-k.
#include "fg_common.cuh"
#include "fg_sampler.cuh"
#include "fg_nucleus.cuh"

namespace fg {

__global__ void philox_uniforms_kernel(uint64_t seed, const int32_t* __restrict__ seq_ids, int32_t n_rows,
                                       int32_t round_idx, const int32_t* __restrict__ round_dev, int32_t n_draws,
                                       float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)n_rows * n_draws) return;
    const int32_t r = (int32_t)(i / n_draws), d = (int32_t)(i % n_draws);
    const int32_t round = round_idx + (round_dev != nullptr ? *round_dev : 0);
    out[i] = philox_uniform(seed, (uint32_t)seq_ids[r], (uint32_t)round, (uint32_t)d);
}

template <typename T>
__global__ void __launch_bounds__(FG_SAMPLE_LANES) sample_rows_kernel(
    const T* __restrict__ logits, int64_t row_stride, int32_t V, const float* __restrict__ uniforms,
    int64_t u_stride, int32_t do_sample, float temperature, float top_p, int32_t top_k,
    const int32_t* __restrict__ forced,
    int32_t* __restrict__ out) {
    __shared__ SampleSmem sm;
    __shared__ NucleusSmem ns;
    const int32_t r = blockIdx.x;
    if (forced != nullptr && forced[r] >= 0) {
        if (threadIdx.x == 0) out[r] = forced[r];
        return;
    }
    const T* row = logits + (int64_t)r * row_stride;
    const float u = uniforms[(int64_t)r * u_stride];
    const int32_t tok = sample_cuts(do_sample, temperature, top_p, top_k, V)
                            ? block_sample_kept<T>(row, V, temperature, top_p, top_k, u, sm, ns)
                            : block_sample<T>(row, V, temperature, do_sample != 0, u, sm);
    if (threadIdx.x == 0) out[r] = tok;
}

// ----------------------------------------------------------------- top-k
__device__ __forceinline__ bool better(float av, int32_t ai, float bv, int32_t bi) {
    return av > bv || (av == bv && ai < bi);
}

// Per-row top-K (value descending, index ascending), row maximum and
// optional logsumexp.  Each thread keeps a sorted K-list of the entries it
// visits (vector loads, four in flight); the lists are merged by K rounds of
// a block-wide "best head" reduction.
template <typename T, int K, int NT, bool LSE>
__global__ void __launch_bounds__(NT) row_topk_kernel(const T* __restrict__ logits, int64_t row_stride, int32_t V,
                                                      int32_t k, int32_t* __restrict__ out_idx,
                                                      float* __restrict__ out_val, float* __restrict__ out_max,
                                                      float* __restrict__ out_lse, int32_t round_lse) {
    __shared__ float sv[NT * K];
    __shared__ int32_t si[NT * K];
    __shared__ float redv[NT / 32];
    __shared__ int32_t redi[NT / 32];
    __shared__ int32_t redt[NT / 32];
    __shared__ float reds[NT / 32];
    __shared__ int32_t winner;
    const int tid = threadIdx.x;
    const T* row = logits + (int64_t)blockIdx.x * row_stride;
    float v[K];
    int32_t id[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
        v[j] = -INFINITY;
        id[j] = 0x7fffffff;
    }
    float m = -INFINITY, s = 0.0f;
    auto visit = [&](float x, int32_t i) {
        if (LSE) {
            if (x > m) {
                s = (m == -INFINITY) ? 0.0f : s * expf(m - x);
                m = x;
            }
            if (x != -INFINITY) s += expf(x - m);
        }
        // indices arrive increasing per thread: an equal value stays behind
        if (better(x, i, v[K - 1], id[K - 1])) {
            float cv = x;
            int32_t ci = i;
#pragma unroll
            for (int j = 0; j < K; ++j) {
                if (better(cv, ci, v[j], id[j])) {
                    const float tv = v[j];
                    const int32_t ti = id[j];
                    v[j] = cv;
                    id[j] = ci;
                    cv = tv;
                    ci = ti;
                }
            }
        }
    };
    if (row_vectorizable<T>(row, V)) {
        constexpr int NV = Vec<T>::N;
        const int32_t nvec = V / NV;
        for (int32_t v0 = tid; v0 < nvec; v0 += 4 * NT) {
            uint4 u[4];
#pragma unroll
            for (int k2 = 0; k2 < 4; ++k2) {
                const int32_t vi = v0 + k2 * NT;
                u[k2] = vi < nvec ? ldg16(row + (int64_t)vi * NV) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int k2 = 0; k2 < 4; ++k2) {
                const int32_t vi = v0 + k2 * NT;
                if (vi >= nvec) break;
                float f[NV];
                unpack<T>(u[k2], f);
#pragma unroll
                for (int e = 0; e < NV; ++e) visit(f[e], vi * NV + e);
            }
        }
    } else {
        for (int32_t i = tid; i < V; i += NT) visit(to_f<T>(row[i]), i);
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
        sv[tid * K + j] = v[j];
        si[tid * K + j] = id[j];
    }
    if (LSE) {
        float gm = warp_max(m);
        if ((tid & 31) == 0) redv[tid >> 5] = gm;
        __syncthreads();
        if (tid < 32) {
            float t = tid < NT / 32 ? redv[tid] : -INFINITY;
            t = warp_max(t);
            if (tid == 0) redv[0] = t;
        }
        __syncthreads();
        gm = redv[0];
        float ls = (m == -INFINITY) ? 0.0f : s * expf(m - gm);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
        if ((tid & 31) == 0) reds[tid >> 5] = ls;
        __syncthreads();
        if (tid == 0) {
            float tot = 0.0f;
            for (int w = 0; w < NT / 32; ++w) tot += reds[w];
            float lse = gm + logf(tot);
            if (round_lse == FG_DTYPE_BF16) lse = __bfloat162float(__float2bfloat16_rn(lse));
            if (round_lse == FG_DTYPE_F16) lse = __half2float(__float2half_rn(lse));
            out_lse[blockIdx.x] = lse;
        }
    }
    __syncthreads();
    // k rounds of "best head among all thread lists"
    int head = 0;
    for (int r = 0; r < k; ++r) {
        float bv = head < K ? sv[tid * K + head] : -INFINITY;
        int32_t bi = head < K ? si[tid * K + head] : 0x7fffffff;
        int bt = tid;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const int ot = __shfl_xor_sync(0xffffffffu, bt, o);
            if (better(ov, oi, bv, bi) || (ov == bv && oi == bi && ot < bt)) {
                bv = ov;
                bi = oi;
                bt = ot;
            }
        }
        if ((tid & 31) == 0) {
            redv[tid >> 5] = bv;
            redi[tid >> 5] = bi;
            redt[tid >> 5] = bt;
        }
        __syncthreads();
        if (tid < 32) {
            float wv = tid < NT / 32 ? redv[tid] : -INFINITY;
            int32_t wi = tid < NT / 32 ? redi[tid] : 0x7fffffff;
            int wt = tid < NT / 32 ? redt[tid] : 0x7fffffff;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, wv, o);
                const int32_t oi = __shfl_xor_sync(0xffffffffu, wi, o);
                const int ot = __shfl_xor_sync(0xffffffffu, wt, o);
                if (better(ov, oi, wv, wi) || (ov == wv && oi == wi && ot < wt)) {
                    wv = ov;
                    wi = oi;
                    wt = ot;
                }
            }
            if (tid == 0) {
                winner = wt;
                out_idx[(int64_t)blockIdx.x * k + r] = (wi == 0x7fffffff) ? 0 : wi;
                out_val[(int64_t)blockIdx.x * k + r] = wv;
                if (r == 0) out_max[blockIdx.x] = wv;
            }
        }
        __syncthreads();
        if (tid == winner) ++head;
    }
}

// Block-wide best (value desc, index asc) of one candidate per thread; every
// thread gets the winner and the winning thread's id.
template <int NT>
__device__ __forceinline__ void block_best_of(float& bv, int32_t& bi, int& bt, float* redv, int32_t* redi,
                                              int32_t* redt) {
    const int tid = threadIdx.x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        const int ot = __shfl_xor_sync(0xffffffffu, bt, o);
        if (better(ov, oi, bv, bi) || (ov == bv && oi == bi && ot < bt)) {
            bv = ov;
            bi = oi;
            bt = ot;
        }
    }
    if ((tid & 31) == 0) {
        redv[tid >> 5] = bv;
        redi[tid >> 5] = bi;
        redt[tid >> 5] = bt;
    }
    __syncthreads();
    bv = redv[0];
    bi = redi[0];
    bt = redt[0];
#pragma unroll
    for (int w = 1; w < NT / 32; ++w)
        if (better(redv[w], redi[w], bv, bi) || (redv[w] == bv && redi[w] == bi && redt[w] < bt)) {
            bv = redv[w];
            bi = redi[w];
            bt = redt[w];
        }
    __syncthreads();
}

// The same per-row top-K without the logsumexp, a row spread over a cluster
// of S CTAs, CTA r on vocabulary slice r (whole 16-byte vectors):
//   pass A  every thread takes the maximum of its entries; tau_r, the k-th
//           largest thread maximum, has k entries of the slice at or above
//           it, so it is at most the row's k-th best value, and so is
//           tau = max_r tau_r (exchanged through distributed shared memory);
//   pass B  the entries >= tau are collected in shared memory -- every
//           entry of the row's top-k is among them -- and the slice's k
//           best candidates are picked by k block-wide reductions.
//           When more than 2 * NT entries tie at or above tau (flat rows),
//           the slice falls back to per-thread sorted lists over all of it;
//   merge   each CTA stores its list into CTA 0 (stores only), which selects
//           the row's k best with one warp.
// The order (value desc, index asc) is total, so the result is the one-CTA
// kernel's bit for bit; NaN never enters (fmaxf skips it, >= is false).
template <typename T, int K, int NT, int S>
__global__ void __launch_bounds__(NT) row_topk_cluster_kernel(const T* __restrict__ logits, int64_t row_stride,
                                                              int32_t V, int32_t k, int32_t* __restrict__ out_idx,
                                                              float* __restrict__ out_val,
                                                              float* __restrict__ out_max) {
    constexpr int CAP = 2 * NT;
    __shared__ float sv[NT * K];      // fallback lists
    __shared__ int32_t si[NT * K];
    __shared__ float tmax[NT];
    __shared__ float cand_v[CAP];
    __shared__ int32_t cand_i[CAP];
    __shared__ int32_t cand_n;
    __shared__ float tau_all[S];
    __shared__ float redv[NT / 32];
    __shared__ int32_t redi[NT / 32];
    __shared__ int32_t redt[NT / 32];
    __shared__ float slice_v[K];
    __shared__ int32_t slice_i[K];
    __shared__ float all_v[S * K];   // CTA 0: every slice's list
    __shared__ int32_t all_i[S * K];
    const int tid = threadIdx.x;
    const uint32_t rank = cl_rank();
    const int64_t r = blockIdx.x / S;
    const T* row = logits + r * row_stride;
    constexpr int NV = Vec<T>::N;
    const int32_t span = ((V + S - 1) / S + NV - 1) / NV * NV;
    const int32_t lo = min(V, (int32_t)rank * span), hi = min(V, lo + span);
    const bool vec = row_vectorizable<T>(row, V);  // then lo and hi are multiples of NV
    const int32_t nvec = vec ? (hi - lo) / NV : 0;
    const T* base = row + lo;
    // ---- pass A: thread maxima, tau_r, tau
    float tm = -INFINITY;
    if (vec) {
        for (int32_t v0 = tid; v0 < nvec; v0 += 4 * NT) {
            uint4 u[4];
#pragma unroll
            for (int k2 = 0; k2 < 4; ++k2) {
                const int32_t vi = v0 + k2 * NT;
                u[k2] = vi < nvec ? ldg16(base + (int64_t)vi * NV) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int k2 = 0; k2 < 4; ++k2) {
                if (v0 + k2 * NT >= nvec) break;
                float f[NV];
                unpack<T>(u[k2], f);
#pragma unroll
                for (int e = 0; e < NV; ++e) tm = fmaxf(tm, f[e]);
            }
        }
    } else {
        for (int32_t i = lo + tid; i < hi; i += NT) tm = fmaxf(tm, to_f<T>(row[i]));
    }
    tmax[tid] = tm;
    if (tid == 0) cand_n = 0;
    __syncthreads();
    if (tid < 32) {
        // k rounds of a warp maximum over the NT thread maxima, one instance
        // removed per round: tau_r is the k-th largest
        constexpr int PER = NT / 32;
        float a[PER];
#pragma unroll
        for (int j = 0; j < PER; ++j) a[j] = tmax[tid + 32 * j];
        float tau = -INFINITY;
        for (int rr = 0; rr < k; ++rr) {
            float lb = a[0];
#pragma unroll
            for (int j = 1; j < PER; ++j) lb = fmaxf(lb, a[j]);
            tau = warp_max(lb);
            const unsigned holders = __ballot_sync(0xffffffffu, lb == tau);
            if (holders != 0u && tid == __ffs(holders) - 1) {
                bool done = false;
#pragma unroll
                for (int j = 0; j < PER; ++j)
                    if (!done && a[j] == tau) {
                        a[j] = -INFINITY;
                        done = true;
                    }
            }
        }
        if (tid < S) cl_st_f32(&tau_all[rank], tid, tau);
    }
    cl_sync();  // every CTA holds every tau_r
    float tau = tau_all[0];
#pragma unroll
    for (int j = 1; j < S; ++j) tau = fmaxf(tau, tau_all[j]);
    // ---- pass B: candidates >= tau
    auto offer = [&](float x, int32_t i) {
        if (x >= tau) {
            const int32_t slot = atomicAdd(&cand_n, 1);
            if (slot < CAP) {
                cand_v[slot] = x;
                cand_i[slot] = i;
            }
        }
    };
    if (vec) {
        for (int32_t v0 = tid; v0 < nvec; v0 += 4 * NT) {
            uint4 u[4];
#pragma unroll
            for (int k2 = 0; k2 < 4; ++k2) {
                const int32_t vi = v0 + k2 * NT;
                u[k2] = vi < nvec ? ldg16(base + (int64_t)vi * NV) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int k2 = 0; k2 < 4; ++k2) {
                const int32_t vi = v0 + k2 * NT;
                if (vi >= nvec) break;
                float f[NV];
                unpack<T>(u[k2], f);
                float vm = f[0];
#pragma unroll
                for (int e = 1; e < NV; ++e) vm = fmaxf(vm, f[e]);
                if (vm >= tau) {
#pragma unroll
                    for (int e = 0; e < NV; ++e) offer(f[e], lo + vi * NV + e);
                }
            }
        }
    } else {
        for (int32_t i = lo + tid; i < hi; i += NT) offer(to_f<T>(row[i]), i);
    }
    __syncthreads();
    const int32_t n_cand = cand_n;
    if (n_cand <= CAP) {
        // the slice's k best candidates: k block-wide reductions
        float c0 = tid < n_cand ? cand_v[tid] : -INFINITY, c1 = tid + NT < n_cand ? cand_v[tid + NT] : -INFINITY;
        int32_t i0 = tid < n_cand ? cand_i[tid] : 0x7fffffff, i1 = tid + NT < n_cand ? cand_i[tid + NT] : 0x7fffffff;
        for (int rr = 0; rr < k; ++rr) {
            const bool second = better(c1, i1, c0, i0);
            float bv = second ? c1 : c0;
            int32_t bi = second ? i1 : i0;
            int bt = tid;
            block_best_of<NT>(bv, bi, bt, redv, redi, redt);
            if (tid == 0) {
                slice_v[rr] = bv;
                slice_i[rr] = bi;
            }
            if (tid == bt) {
                if (second) {
                    c1 = -INFINITY;
                    i1 = 0x7fffffff;
                } else {
                    c0 = -INFINITY;
                    i0 = 0x7fffffff;
                }
            }
        }
    } else {
        // many entries tied at or above tau: per-thread sorted lists over the
        // whole slice, merged by k block-wide rounds
        float v[K];
        int32_t id[K];
#pragma unroll
        for (int j = 0; j < K; ++j) {
            v[j] = -INFINITY;
            id[j] = 0x7fffffff;
        }
        auto visit = [&](float x, int32_t i) {
            if (better(x, i, v[K - 1], id[K - 1])) {
                float cv = x;
                int32_t ci = i;
#pragma unroll
                for (int j = 0; j < K; ++j) {
                    if (better(cv, ci, v[j], id[j])) {
                        const float tv = v[j];
                        const int32_t ti = id[j];
                        v[j] = cv;
                        id[j] = ci;
                        cv = tv;
                        ci = ti;
                    }
                }
            }
        };
        if (vec) {
            for (int32_t vi = tid; vi < nvec; vi += NT) {
                float f[NV];
                unpack<T>(ldg16(base + (int64_t)vi * NV), f);
#pragma unroll
                for (int e = 0; e < NV; ++e) visit(f[e], lo + vi * NV + e);
            }
        } else {
            for (int32_t i = lo + tid; i < hi; i += NT) visit(to_f<T>(row[i]), i);
        }
#pragma unroll
        for (int j = 0; j < K; ++j) {
            sv[tid * K + j] = v[j];
            si[tid * K + j] = id[j];
        }
        __syncthreads();
        int head = 0;
        for (int rr = 0; rr < k; ++rr) {
            float bv = head < K ? sv[tid * K + head] : -INFINITY;
            int32_t bi = head < K ? si[tid * K + head] : 0x7fffffff;
            int bt = tid;
            block_best_of<NT>(bv, bi, bt, redv, redi, redt);
            if (tid == 0) {
                slice_v[rr] = bv;
                slice_i[rr] = bi;
            }
            if (tid == bt) ++head;
        }
    }
    __syncthreads();
    // push this slice's list into CTA 0 (stores only: nobody reads a peer's
    // memory, so a CTA may exit as soon as the barrier below completes)
    if (tid < k) {
        cl_st_f32(&all_v[rank * K + tid], 0, slice_v[tid]);
        cl_st_s32(&all_i[rank * K + tid], 0, slice_i[tid]);
    }
    cl_sync();  // CTA 0 holds every slice list
    if (rank == 0 && tid < 32) {
        // k rounds of a warp-wide best over the S * k candidates (lane l holds
        // slots l, l + 32, ...), the winner's slot retired after each round
        constexpr int PER = (S * K + 31) / 32;
        float cv[PER];
        int32_t ci[PER];
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int c = tid + 32 * j;
            const bool live = c < S * K && (c % K) < k;
            cv[j] = live ? all_v[c] : -INFINITY;
            ci[j] = live ? all_i[c] : 0x7fffffff;
        }
        for (int rr = 0; rr < k; ++rr) {
            int bj = 0;
#pragma unroll
            for (int j = 1; j < PER; ++j)
                if (better(cv[j], ci[j], cv[bj], ci[bj])) bj = j;
            float bv = cv[0];
            int32_t bi = ci[0];
#pragma unroll
            for (int j = 1; j < PER; ++j)
                if (j == bj) {
                    bv = cv[j];
                    bi = ci[j];
                }
            int bl = tid;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
                const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
                if (better(ov, oi, bv, bi) || (ov == bv && oi == bi && ol < bl)) {
                    bv = ov;
                    bi = oi;
                    bl = ol;
                }
            }
            if (tid == 0) {
                out_idx[r * k + rr] = (bi == 0x7fffffff) ? 0 : bi;
                out_val[r * k + rr] = bv;
                if (rr == 0) out_max[r] = bv;
            }
            if (tid == bl) {
#pragma unroll
                for (int j = 0; j < PER; ++j)
                    if (j == bj) {
                        cv[j] = -INFINITY;
                        ci[j] = 0x7fffffff;
                    }
            }
        }
    }
}

template <int S, typename T, typename KernelT>
static cudaError_t launch_cluster(KernelT kernel, int32_t n_rows, int nt, cudaStream_t st, const T* logits,
                                  int64_t row_stride, int32_t V, int32_t k, int32_t* idx, float* val, float* mx) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)n_rows * S);
    cfg.blockDim = dim3(nt);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, logits, row_stride, V, k, idx, val, mx);
}

// Rows spread over 8-CTA clusters (no logsumexp requested).
constexpr int kTopkClusterCtas = 8;

template <typename T>
static void launch_topk_cluster(const T* logits, int64_t row_stride, int32_t V, int32_t n_rows, int32_t k, int32_t* idx,
                                float* val, float* mx, cudaStream_t st) {
    constexpr int S = kTopkClusterCtas;
    if (k <= 1)
        launch_cluster<S>(row_topk_cluster_kernel<T, 1, 256, S>, n_rows, 256, st, logits, row_stride, V, k, idx, val, mx);
    else if (k <= 2)
        launch_cluster<S>(row_topk_cluster_kernel<T, 2, 256, S>, n_rows, 256, st, logits, row_stride, V, k, idx, val, mx);
    else if (k <= 4)
        launch_cluster<S>(row_topk_cluster_kernel<T, 4, 256, S>, n_rows, 256, st, logits, row_stride, V, k, idx, val, mx);
    else if (k <= 8)
        launch_cluster<S>(row_topk_cluster_kernel<T, 8, 128, S>, n_rows, 128, st, logits, row_stride, V, k, idx, val, mx);
    else
        launch_cluster<S>(row_topk_cluster_kernel<T, 16, 64, S>, n_rows, 64, st, logits, row_stride, V, k, idx, val, mx);
}

template <typename T, bool LSE>
static void launch_topk(const T* logits, int64_t row_stride, int32_t V, int32_t n_rows, int32_t k, int32_t* idx,
                        float* val, float* mx, float* lse, int32_t dtype, cudaStream_t st) {
    if (k <= 1)
        row_topk_kernel<T, 1, 1024, LSE><<<n_rows, 1024, 0, st>>>(logits, row_stride, V, k, idx, val, mx, lse, dtype);
    else if (k <= 2)
        row_topk_kernel<T, 2, 1024, LSE><<<n_rows, 1024, 0, st>>>(logits, row_stride, V, k, idx, val, mx, lse, dtype);
    else if (k <= 4)
        row_topk_kernel<T, 4, 1024, LSE><<<n_rows, 1024, 0, st>>>(logits, row_stride, V, k, idx, val, mx, lse, dtype);
    else if (k <= 8)
        row_topk_kernel<T, 8, 512, LSE><<<n_rows, 512, 0, st>>>(logits, row_stride, V, k, idx, val, mx, lse, dtype);
    else
        row_topk_kernel<T, 16, 256, LSE><<<n_rows, 256, 0, st>>>(logits, row_stride, V, k, idx, val, mx, lse, dtype);
}

template <typename T>
static void dispatch_topk(const void* logits, int64_t row_stride, int32_t V, int32_t n_rows, int32_t k, int32_t* idx,
                          float* val, float* mx, float* lse, int32_t dtype, cudaStream_t st) {
    if (lse)
        launch_topk<T, true>((const T*)logits, row_stride, V, n_rows, k, idx, val, mx, lse, dtype, st);
    else
        launch_topk_cluster<T>((const T*)logits, row_stride, V, n_rows, k, idx, val, mx, st);
}

}  // namespace fg

using namespace fg;

extern "C" fg_status fg_philox_uniforms(uint64_t seed, const int32_t* seq_ids, int32_t n_rows, int32_t round_idx,
                                        const int32_t* round_dev, int32_t n_draws, float* out, void* stream) {
    if (n_rows < 0 || n_draws < 0 || (n_rows > 0 && n_draws > 0 && (!seq_ids || !out))) return FG_EINVAL;
    const int64_t n = (int64_t)n_rows * n_draws;
    if (n == 0) return FG_OK;
    philox_uniforms_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        seed, seq_ids, n_rows, round_idx, round_dev, n_draws, out);
    return launch_status();
}

extern "C" fg_status fg_sample_rows(const void* logits, int32_t dtype, int64_t row_stride, int32_t vocab,
                                    int32_t n_rows, const float* uniforms, int64_t u_stride, int32_t do_sample,
                                    float temperature, float top_p, int32_t top_k, const int32_t* forced,
                                    int32_t* out_tokens, void* stream) {
    if (n_rows == 0) return FG_OK;
    if (!logits || !uniforms || !out_tokens || vocab <= 0 || n_rows < 0 || row_stride < vocab) return FG_EINVAL;
    cudaStream_t st = (cudaStream_t)stream;
    switch (dtype) {
        case FG_DTYPE_F32:
            sample_rows_kernel<float><<<n_rows, FG_SAMPLE_LANES, 0, st>>>(
                (const float*)logits, row_stride, vocab, uniforms, u_stride, do_sample, temperature, top_p, top_k,
                forced, out_tokens);
            break;
        case FG_DTYPE_BF16:
            sample_rows_kernel<__nv_bfloat16><<<n_rows, FG_SAMPLE_LANES, 0, st>>>(
                (const __nv_bfloat16*)logits, row_stride, vocab, uniforms, u_stride, do_sample, temperature, top_p, top_k,
                forced, out_tokens);
            break;
        case FG_DTYPE_F16:
            sample_rows_kernel<__half><<<n_rows, FG_SAMPLE_LANES, 0, st>>>(
                (const __half*)logits, row_stride, vocab, uniforms, u_stride, do_sample, temperature, top_p, top_k,
                forced, out_tokens);
            break;
        default:
            return FG_EINVAL;
    }
    return launch_status();
}

extern "C" fg_status fg_row_topk(const void* logits, int32_t dtype, int64_t row_stride, int32_t vocab,
                                 int32_t n_rows, int32_t k, int32_t* out_idx, float* out_val, float* out_max,
                                 float* out_lse, void* stream) {
    if (n_rows == 0) return FG_OK;
    if (!logits || !out_idx || !out_val || !out_max || vocab <= 0 || row_stride < vocab) return FG_EINVAL;
    if (k <= 0 || k > FG_MAX_TOPK || k > vocab) return FG_ECAPACITY;
    cudaStream_t st = (cudaStream_t)stream;
    switch (dtype) {
        case FG_DTYPE_F32:
            dispatch_topk<float>(logits, row_stride, vocab, n_rows, k, out_idx, out_val, out_max, out_lse, dtype, st);
            break;
        case FG_DTYPE_BF16:
            dispatch_topk<__nv_bfloat16>(logits, row_stride, vocab, n_rows, k, out_idx, out_val, out_max, out_lse,
                                         dtype, st);
            break;
        case FG_DTYPE_F16:
            dispatch_topk<__half>(logits, row_stride, vocab, n_rows, k, out_idx, out_val, out_max, out_lse, dtype, st);
            break;
        default:
            return FG_EINVAL;
    }
    return launch_status();
}

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
    int64_t u_stride, int32_t do_sample, float temperature, float top_p, const int32_t* __restrict__ forced,
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
    const bool nucleus = do_sample != 0 && temperature != 0.0f && top_p > 0.0f && top_p < 1.0f;
    const int32_t tok = nucleus ? block_sample_nucleus<T>(row, V, temperature, top_p, u, sm, ns)
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
        launch_topk<T, false>((const T*)logits, row_stride, V, n_rows, k, idx, val, mx, lse, dtype, st);
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
                                    float temperature, float top_p, const int32_t* forced, int32_t* out_tokens,
                                    void* stream) {
    if (n_rows == 0) return FG_OK;
    if (!logits || !uniforms || !out_tokens || vocab <= 0 || n_rows < 0 || row_stride < vocab) return FG_EINVAL;
    cudaStream_t st = (cudaStream_t)stream;
    switch (dtype) {
        case FG_DTYPE_F32:
            sample_rows_kernel<float><<<n_rows, FG_SAMPLE_LANES, 0, st>>>(
                (const float*)logits, row_stride, vocab, uniforms, u_stride, do_sample, temperature, top_p, forced,
                out_tokens);
            break;
        case FG_DTYPE_BF16:
            sample_rows_kernel<__nv_bfloat16><<<n_rows, FG_SAMPLE_LANES, 0, st>>>(
                (const __nv_bfloat16*)logits, row_stride, vocab, uniforms, u_stride, do_sample, temperature, top_p, forced,
                out_tokens);
            break;
        case FG_DTYPE_F16:
            sample_rows_kernel<__half><<<n_rows, FG_SAMPLE_LANES, 0, st>>>(
                (const __half*)logits, row_stride, vocab, uniforms, u_stride, do_sample, temperature, top_p, forced,
                out_tokens);
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

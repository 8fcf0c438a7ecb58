// fg_layers.cu -- elementwise pieces of the verify forward and the MEDUSA heads.
//
// Half-precision variants round after each step the way the reference's
// PyTorch arithmetic does (every bf16 tensor op rounds its result), so the
// verify forward tracks the reference within bf16 tolerance; the f32
// variants stay in f32.
#include "fg_common.cuh"

namespace fg {

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

template <typename T>
__device__ __forceinline__ float tf(T v);
template <>
__device__ __forceinline__ float tf<float>(float v) { return v; }
template <>
__device__ __forceinline__ float tf<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float tf<__half>(__half v) { return __half2float(v); }

// rounds v to T and back (identity for float)
template <typename T>
__device__ __forceinline__ float rnd(float v) { return tf<T>(from_f<T>(v)); }

// --------------------------------------------------------------- RoPE + KV
// One rotation pair as the reference evaluates q*cos + rotate_half(q)*sin:
// each product and the sum rounded separately (no fused multiply-add), then
// rounded to the activation dtype.
template <typename T>
__device__ __forceinline__ void rope_pair(float a, float b, float c, float s, float& o1, float& o2) {
    o1 = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(a, c)), rnd<T>(__fmul_rn(-b, s))));
    o2 = rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(b, c)), rnd<T>(__fmul_rn(a, s))));
}

// One CTA per (row, node); threads over (head, pair).  HF computes
// cos/sin(pos * inv_freq) in fp32, casts them to the activation dtype and
// evaluates q*cos + rotate_half(q)*sin in that dtype.
template <typename T>
__global__ void rope_kv_kernel(const T* __restrict__ qkv, const int32_t* __restrict__ positions,
                               const float* __restrict__ inv_freq, float attn_scaling, int32_t n_nodes, int32_t Hq,
                               int32_t Hkv, int32_t D, const int32_t* __restrict__ kv_len, T* __restrict__ kc,
                               T* __restrict__ vc, int64_t sb, int64_t sh, int64_t ss, int32_t cap,
                               const int32_t* __restrict__ kv_rows, int32_t kv_batch, T* __restrict__ q_out) {
    __shared__ float cs[2][128];  // cos / sin per frequency, once per token
    // the tree attention that follows may start its prefix loads now; it
    // waits for this grid to finish before reading Q or the tree K/V
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int32_t tokn = blockIdx.x;  // b * n_nodes + node
    const int32_t b = tokn / n_nodes, node = tokn % n_nodes;
    const float pos = (float)positions[tokn];
    const int32_t half = D / 2;
    const T* src = qkv + (int64_t)tokn * (Hq + 2 * Hkv) * D;
    const int32_t slotpos = kv_len[b] + node;
    const int32_t bk = cache_row(kv_rows, kv_batch, b);
    const bool in_cap = slotpos < cap && bk >= 0;
    for (int32_t i = threadIdx.x; i < half; i += blockDim.x) {
        const float f = __fmul_rn(pos, inv_freq[i]);
        float c = cosf(f), s = sinf(f);
        if (attn_scaling != 1.0f) {
            c = c * attn_scaling;
            s = s * attn_scaling;
        }
        cs[0][i] = rnd<T>(c);
        cs[1][i] = rnd<T>(s);
    }
    __syncthreads();
    for (int32_t e = threadIdx.x; e < (Hq + Hkv) * half; e += blockDim.x) {
        const int32_t h = e / half, i = e % half;
        const float c = cs[0][i], s = cs[1][i];
        const T* x = src + (int64_t)h * D;
        const float x1 = tf<T>(x[i]), x2 = tf<T>(x[i + half]);
        // out[i] = x1*c - x2*s ; out[i+half] = x2*c + x1*s  (each product rounded)
        float o1, o2;
        rope_pair<T>(x1, x2, c, s, o1, o2);
        if (h < Hq) {
            T* qo = q_out + ((int64_t)tokn * Hq + h) * D;
            qo[i] = from_f<T>(o1);
            qo[i + half] = from_f<T>(o2);
        } else if (in_cap) {
            const int32_t kh = h - Hq;
            T* ko = kc + (int64_t)bk * sb + (int64_t)kh * sh + (int64_t)slotpos * ss;
            ko[i] = from_f<T>(o1);
            ko[i + half] = from_f<T>(o2);
        }
    }
    if (in_cap)
        for (int32_t e = threadIdx.x; e < Hkv * D; e += blockDim.x) {
            const int32_t kh = e / D, d = e % D;
            vc[(int64_t)bk * sb + (int64_t)kh * sh + (int64_t)slotpos * ss + d] = src[(int64_t)(Hq + Hkv + kh) * D + d];
        }
}

// cos/sin(pos * inv_freq) * scaling rounded to the activation dtype, once per
// round: [2][n_tokens][half] (cos rows, then sin rows).  Positions are the
// same for every layer of a round, so the layers share one table.
template <typename T>
__global__ void rope_table_kernel(const int32_t* __restrict__ positions, int32_t n_tokens,
                                  const float* __restrict__ inv_freq, int32_t half, float attn_scaling,
                                  T* __restrict__ cs) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (int64_t)n_tokens * half) return;
    const int32_t t = (int32_t)(e / half), i = (int32_t)(e % half);
    const float f = __fmul_rn((float)positions[t], inv_freq[i]);
    float c = cosf(f), s = sinf(f);
    if (attn_scaling != 1.0f) {
        c = c * attn_scaling;
        s = s * attn_scaling;
    }
    cs[e] = from_f<T>(c);
    cs[(int64_t)n_tokens * half + e] = from_f<T>(s);
}

// RoPE + tree K/V write from a cos/sin table: one CTA per (row, node), one
// thread per 8 consecutive rotation pairs of a head (16-byte vectors), the
// same roundings as rope_kv_kernel.
template <typename T>
__global__ void __launch_bounds__(128) rope_kv_table_kernel(
    const T* __restrict__ qkv, const T* __restrict__ cs, int32_t n_tokens, int32_t n_nodes, int32_t Hq, int32_t Hkv,
    int32_t D, const int32_t* __restrict__ kv_len, T* __restrict__ kc, T* __restrict__ vc, int64_t sb, int64_t sh,
    int64_t ss, int32_t cap, const int32_t* __restrict__ kv_rows, int32_t kv_batch, T* __restrict__ q_out) {
    // qkv comes from the projection before; the tree attention after may then
    // start (its prefix loads), waiting for this grid before reading Q or the tree K/V
    pdl_wait_then_release();
    constexpr int NV = 16 / sizeof(T);
    const int32_t tokn = blockIdx.x;
    const int32_t b = tokn / n_nodes, node = tokn % n_nodes;
    const int32_t half = D / 2, vph = half / NV;  // vectors per half-head
    const T* src = qkv + (int64_t)tokn * (Hq + 2 * Hkv) * D;
    const int32_t slotpos = kv_len[b] + node;
    const int32_t bk = cache_row(kv_rows, kv_batch, b);
    const bool in_cap = slotpos < cap && bk >= 0;
    const T* cr = cs + (int64_t)tokn * half;
    const T* sr = cs + ((int64_t)n_tokens + tokn) * half;
    for (int32_t e = threadIdx.x; e < (Hq + Hkv) * vph; e += blockDim.x) {
        const int32_t h = e / vph, i = (e % vph) * NV;
        const T* x = src + (int64_t)h * D;
        const uint4 u1 = *reinterpret_cast<const uint4*>(x + i), u2 = *reinterpret_cast<const uint4*>(x + i + half);
        const uint4 uc = *reinterpret_cast<const uint4*>(cr + i), us = *reinterpret_cast<const uint4*>(sr + i);
        const T *x1 = reinterpret_cast<const T*>(&u1), *x2 = reinterpret_cast<const T*>(&u2);
        const T *cc = reinterpret_cast<const T*>(&uc), *sv = reinterpret_cast<const T*>(&us);
        uint4 r1, r2;
        T *o1 = reinterpret_cast<T*>(&r1), *o2 = reinterpret_cast<T*>(&r2);
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            float v1, v2;
            rope_pair<T>(tf<T>(x1[k]), tf<T>(x2[k]), tf<T>(cc[k]), tf<T>(sv[k]), v1, v2);
            o1[k] = from_f<T>(v1);
            o2[k] = from_f<T>(v2);
        }
        T* dst = nullptr;
        if (h < Hq) {
            dst = q_out + ((int64_t)tokn * Hq + h) * D;
        } else if (in_cap) {
            dst = kc + (int64_t)bk * sb + (int64_t)(h - Hq) * sh + (int64_t)slotpos * ss;
        }
        if (dst) {
            *reinterpret_cast<uint4*>(dst + i) = r1;
            *reinterpret_cast<uint4*>(dst + i + half) = r2;
        }
    }
    if (in_cap)
        for (int32_t e = threadIdx.x; e < Hkv * (D / NV); e += blockDim.x) {
            const int32_t kh = e / (D / NV), d = (e % (D / NV)) * NV;
            *reinterpret_cast<uint4*>(vc + (int64_t)bk * sb + (int64_t)kh * sh + (int64_t)slotpos * ss + d) =
                *reinterpret_cast<const uint4*>(src + (int64_t)(Hq + Hkv + kh) * D + d);
        }
}

// ---------------------------------------------------------------- norms
template <typename T>
__device__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < nw; ++i) t += red[i];
    __syncthreads();
    return t;
}

// Vectorized RMSNorm: 128 threads, rows of up to 128 * 4 vectors kept in
// registers between the sum of squares and the scaling.
template <typename T>
__global__ void __launch_bounds__(128) rmsnorm_vec_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                          int32_t dim, float eps, T* __restrict__ y) {
    pdl_wait_then_release();
    constexpr int NV = 16 / sizeof(T);
    __shared__ float red[32];
    const int32_t nvec = dim / NV;
    const T* xr = x + (int64_t)blockIdx.x * dim;
    uint4 u[4];
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int32_t vi = threadIdx.x + k * 128;
        u[k] = vi < nvec ? *reinterpret_cast<const uint4*>(xr + vi * NV) : make_uint4(0, 0, 0, 0);
        const T* e = reinterpret_cast<const T*>(&u[k]);
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const float v = tf<T>(e[j]);
            ss += v * v;
        }
    }
    ss = block_sum<T>(ss, red);
    const float r = rsqrtf(ss / (float)dim + eps);
    T* yr = y + (int64_t)blockIdx.x * dim;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int32_t vi = threadIdx.x + k * 128;
        if (vi >= nvec) break;
        const uint4 uw = *reinterpret_cast<const uint4*>(w + vi * NV);
        const T* e = reinterpret_cast<const T*>(&u[k]);
        const T* we = reinterpret_cast<const T*>(&uw);
        uint4 res;
        T* o = reinterpret_cast<T*>(&res);
#pragma unroll
        for (int j = 0; j < NV; ++j) o[j] = from_f<T>(tf<T>(we[j]) * rnd<T>(tf<T>(e[j]) * r));
        *reinterpret_cast<uint4*>(yr + vi * NV) = res;
    }
}

template <typename T>
__global__ void rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ w, int32_t dim, float eps,
                               T* __restrict__ y) {
    __shared__ float red[32];
    const T* xr = x + (int64_t)blockIdx.x * dim;
    float ss = 0.0f;
    for (int32_t i = threadIdx.x; i < dim; i += blockDim.x) {
        const float v = tf<T>(xr[i]);
        ss += v * v;
    }
    ss = block_sum<T>(ss, red);
    const float r = rsqrtf(ss / (float)dim + eps);
    T* yr = y + (int64_t)blockIdx.x * dim;
    for (int32_t i = threadIdx.x; i < dim; i += blockDim.x)
        yr[i] = from_f<T>(tf<T>(w[i]) * rnd<T>(tf<T>(xr[i]) * r));
}

template <typename T>
__global__ void layernorm_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ bias,
                                 int32_t dim, float eps, T* __restrict__ y) {
    __shared__ float red[32];
    const T* xr = x + (int64_t)blockIdx.x * dim;
    float s = 0.0f;
    for (int32_t i = threadIdx.x; i < dim; i += blockDim.x) s += tf<T>(xr[i]);
    const float mean = block_sum<T>(s, red) / (float)dim;
    float v = 0.0f;
    for (int32_t i = threadIdx.x; i < dim; i += blockDim.x) {
        const float d = tf<T>(xr[i]) - mean;
        v += d * d;
    }
    const float r = rsqrtf(block_sum<T>(v, red) / (float)dim + eps);
    T* yr = y + (int64_t)blockIdx.x * dim;
    for (int32_t i = threadIdx.x; i < dim; i += blockDim.x)
        yr[i] = from_f<T>((tf<T>(xr[i]) - mean) * r * tf<T>(w[i]) + tf<T>(bias[i]));
}

// ---------------------------------------------------------- activations
// v * sigmoid(v) in fp32 with the fast exponential and division intrinsics;
// the result is rounded to the activation dtype like the reference's, so the
// few-ulp fp32 difference rarely reaches the rounded value.  Large negative v:
// exp overflows to inf and the quotient is -0.
__device__ __forceinline__ float silu(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

// One CTA per row (no index division), 16-byte vectors of gate and up.
template <typename T>
__global__ void __launch_bounds__(256) silu_mul_rows_kernel(const T* __restrict__ gu, int32_t inter,
                                                            T* __restrict__ out) {
    constexpr int NV = 16 / sizeof(T);
    const int64_t r = blockIdx.x;
    const T* g_row = gu + r * 2 * inter;
    const T* u_row = g_row + inter;
    T* o_row = out + r * inter;
    for (int32_t i = threadIdx.x * NV; i < inter; i += blockDim.x * NV) {
        const uint4 ug = *reinterpret_cast<const uint4*>(g_row + i);
        const uint4 uu = *reinterpret_cast<const uint4*>(u_row + i);
        const T* g = reinterpret_cast<const T*>(&ug);
        const T* u = reinterpret_cast<const T*>(&uu);
        uint4 res;
        T* o = reinterpret_cast<T*>(&res);
#pragma unroll
        for (int k = 0; k < NV; ++k) o[k] = from_f<T>(rnd<T>(silu(tf<T>(g[k]))) * tf<T>(u[k]));
        *reinterpret_cast<uint4*>(o_row + i) = res;
    }
}

template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ gu, int32_t inter, int64_t total, T* __restrict__ out) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / inter, i = e % inter;
        const float g = tf<T>(gu[r * 2 * inter + i]), u = tf<T>(gu[r * 2 * inter + inter + i]);
        out[e] = from_f<T>(rnd<T>(silu(g)) * u);
    }
}

template <typename T>
__global__ void silu_residual_kernel(const T* __restrict__ x, const T* __restrict__ y, int64_t n,
                                     T* __restrict__ out) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x)
        out[e] = from_f<T>(tf<T>(x[e]) + rnd<T>(silu(tf<T>(y[e]))));
}

__global__ void gather_rows_kernel(const uint8_t* __restrict__ src, int64_t src_stride, const int32_t* __restrict__ idx,
                                   int64_t row_bytes, uint8_t* __restrict__ out, int64_t out_stride) {
    pdl_wait_then_release();
    const int32_t r = blockIdx.x;
    const uint8_t* s = src + (int64_t)idx[r] * src_stride;
    uint8_t* d = out + (int64_t)r * out_stride;
    for (int64_t o = (int64_t)threadIdx.x * 16; o < row_bytes; o += (int64_t)blockDim.x * 16)
        *reinterpret_cast<uint4*>(d + o) = *reinterpret_cast<const uint4*>(s + o);
}

inline int grid_for(int64_t n) {
    const int64_t g = (n + 255) / 256;
    return (int)(g < 148 * 16 ? g : 148 * 16);
}

}  // namespace fg

using namespace fg;

#define FG_DISPATCH(dtype, CALL)                              \
    switch (dtype) {                                          \
        case FG_DTYPE_F32: { using T = float; CALL; break; }  \
        case FG_DTYPE_BF16: { using T = __nv_bfloat16; CALL; break; } \
        case FG_DTYPE_F16: { using T = __half; CALL; break; } \
        default: return FG_EINVAL;                            \
    }

extern "C" fg_status fg_rope_table(const int32_t* positions, int32_t n_tokens, const float* inv_freq, int32_t half,
                                   float attention_scaling, int32_t dtype, void* cos_sin, void* stream) {
    if (n_tokens == 0) return FG_OK;
    if (!positions || !inv_freq || !cos_sin || n_tokens < 0 || half <= 0) return FG_EINVAL;
    const int64_t n = (int64_t)n_tokens * half;
    cudaStream_t st = (cudaStream_t)stream;
    FG_DISPATCH(dtype, (rope_table_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
                            positions, n_tokens, inv_freq, half, attention_scaling, (T*)cos_sin)));
    return launch_status();
}

extern "C" fg_status fg_rope_kv_write(const void* qkv, int32_t dtype, const int32_t* positions, const float* inv_freq,
                                      float attention_scaling, int32_t B, int32_t n_nodes, int32_t n_q_heads,
                                      int32_t n_kv_heads, int32_t head_dim, const int32_t* kv_len,
                                      const fg_kv_layer* kv, void* q_out, const void* cos_sin, void* stream) {
    if (B * n_nodes == 0) return FG_OK;
    if (!qkv || !positions || !inv_freq || !kv_len || !kv || !kv->k || !kv->v || !q_out || head_dim % 2) return FG_EINVAL;
    if (head_dim > 256) return FG_ECAPACITY;
    cudaStream_t st = (cudaStream_t)stream;
    const int esz = dtype == FG_DTYPE_F32 ? 4 : 2;
    const bool vec = cos_sin != nullptr && ((head_dim / 2) * esz) % 16 == 0 && ((uintptr_t)qkv % 16) == 0 &&
                     ((uintptr_t)q_out % 16) == 0 && ((uintptr_t)cos_sin % 16) == 0 && ((uintptr_t)kv->k % 16) == 0 &&
                     ((uintptr_t)kv->v % 16) == 0 && (kv->stride_s * esz) % 16 == 0 && (kv->stride_h * esz) % 16 == 0 &&
                     (kv->stride_b * esz) % 16 == 0;
    if (vec) {
        cudaError_t e = cudaSuccess;
        FG_DISPATCH(dtype, (e = launch_pdl(rope_kv_table_kernel<T>, dim3(B * n_nodes), dim3(128), 0, st,
                                           (const T*)qkv, (const T*)cos_sin, B * n_nodes, n_nodes, n_q_heads,
                                           n_kv_heads, head_dim, kv_len, (T*)kv->k, (T*)kv->v, kv->stride_b,
                                           kv->stride_h, kv->stride_s, kv->capacity, kv->rows, kv->batch,
                                           (T*)q_out)));
        if (e != cudaSuccess) {
            set_cuda_error(e);
            return FG_ECUDA;
        }
        return launch_status();
    }
    FG_DISPATCH(dtype, (rope_kv_kernel<T><<<B * n_nodes, 128, 0, st>>>(
                            (const T*)qkv, positions, inv_freq, attention_scaling, n_nodes, n_q_heads, n_kv_heads,
                            head_dim, kv_len, (T*)kv->k, (T*)kv->v, kv->stride_b, kv->stride_h, kv->stride_s,
                            kv->capacity, kv->rows, kv->batch, (T*)q_out)));
    return launch_status();
}

extern "C" fg_status fg_rmsnorm(const void* x, const void* weight, int32_t dtype, int32_t n_rows, int32_t dim, float eps,
                                void* y, void* stream) {
    if (n_rows == 0) return FG_OK;
    if (!x || !weight || !y || dim <= 0) return FG_EINVAL;
    cudaStream_t st = (cudaStream_t)stream;
    const int esz = dtype == FG_DTYPE_F32 ? 4 : 2;
    const bool vec = (dim * esz) % 16 == 0 && dim * esz <= 128 * 4 * 16 && ((uintptr_t)x % 16) == 0 &&
                     ((uintptr_t)y % 16) == 0 && ((uintptr_t)weight % 16) == 0;
    if (vec) {
        cudaError_t e = cudaSuccess;
        FG_DISPATCH(dtype, (e = launch_pdl(rmsnorm_vec_kernel<T>, dim3(n_rows), dim3(128), 0, st, (const T*)x,
                                           (const T*)weight, dim, eps, (T*)y)));
        if (e != cudaSuccess) {
            set_cuda_error(e);
            return FG_ECUDA;
        }
    } else {
        FG_DISPATCH(dtype, (rmsnorm_kernel<T><<<n_rows, 256, 0, st>>>((const T*)x, (const T*)weight, dim, eps,
                                                                      (T*)y)));
    }
    return launch_status();
}

extern "C" fg_status fg_layernorm(const void* x, const void* weight, const void* bias, int32_t dtype, int32_t n_rows,
                                  int32_t dim, float eps, void* y, void* stream) {
    if (n_rows == 0) return FG_OK;
    if (!x || !weight || !bias || !y || dim <= 0) return FG_EINVAL;
    cudaStream_t st = (cudaStream_t)stream;
    FG_DISPATCH(dtype, (layernorm_kernel<T><<<n_rows, 256, 0, st>>>((const T*)x, (const T*)weight, (const T*)bias,
                                                                   dim, eps, (T*)y)));
    return launch_status();
}

extern "C" fg_status fg_silu_mul(const void* gu, int32_t dtype, int32_t n_rows, int32_t inter, void* out, void* stream) {
    const int64_t total = (int64_t)n_rows * inter;
    if (total == 0) return FG_OK;
    if (!gu || !out) return FG_EINVAL;
    cudaStream_t st = (cudaStream_t)stream;
    const int esz = dtype == FG_DTYPE_F32 ? 4 : 2;
    if ((inter * esz) % 16 == 0 && ((uintptr_t)gu % 16) == 0 && ((uintptr_t)out % 16) == 0) {
        FG_DISPATCH(dtype, (silu_mul_rows_kernel<T><<<n_rows, 256, 0, st>>>((const T*)gu, inter, (T*)out)));
    } else {
        FG_DISPATCH(dtype, (silu_mul_kernel<T><<<grid_for(total), 256, 0, st>>>((const T*)gu, inter, total, (T*)out)));
    }
    return launch_status();
}

extern "C" fg_status fg_silu_residual(const void* x, const void* y, int32_t dtype, int64_t n, void* out, void* stream) {
    if (n == 0) return FG_OK;
    if (!x || !y || !out) return FG_EINVAL;
    cudaStream_t st = (cudaStream_t)stream;
    FG_DISPATCH(dtype, (silu_residual_kernel<T><<<grid_for(n), 256, 0, st>>>((const T*)x, (const T*)y, n, (T*)out)));
    return launch_status();
}

extern "C" fg_status fg_gather_rows(const void* src, int64_t src_row_stride_bytes, const int32_t* idx, int32_t n_rows,
                                    int64_t row_bytes, void* out, int64_t out_row_stride_bytes, void* stream) {
    if (n_rows == 0) return FG_OK;
    if (!src || !idx || !out || row_bytes <= 0) return FG_EINVAL;
    if (row_bytes % 16 || src_row_stride_bytes % 16 || out_row_stride_bytes % 16 || ((uintptr_t)src % 16) ||
        ((uintptr_t)out % 16))
        return FG_EINVAL;
    const cudaError_t e = launch_pdl(gather_rows_kernel, dim3(n_rows), dim3(128), 0, (cudaStream_t)stream,
                                     (const uint8_t*)src, src_row_stride_bytes, idx, row_bytes, (uint8_t*)out,
                                     out_row_stride_bytes);
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return FG_ECUDA;
    }
    return launch_status();
}

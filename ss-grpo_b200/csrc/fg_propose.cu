// fg_propose.cu -- fg_medusa_propose: the MEDUSA proposal step of a round in
// one call.
//
// Launches: one LayerNorm over the root rows for all heads (the row
// statistics are shared, each head applies its own weight and bias), one
// split-K tcgen05 fc GEMM per head (the lm_head kernel's partial-sum form:
// the H x H weight is read by a full wave of CTAs, each over a k range), one
// pass that adds the partial sums and the bias and applies the SiLU residual
// for all heads' rows, then the tied lm_head over the root and head rows with
// the top-k fused.  Everything in bf16 with the reference's rounding points:
// layer_norm, linear (+bias), silu and the residual add each round their
// result, as MedusaPredictionHead.project_hidden (flashgrpo_b200/models/
// medusa_heads.py:240-244) does in the heads' dtype.
#include "fg_common.cuh"

namespace fg {
namespace prop {

constexpr int kHeadsPerLaunch = 8;

struct HeadNorms {
    const __nv_bfloat16* w[kHeadsPerLaunch];
    const __nv_bfloat16* b[kHeadsPerLaunch];
};

struct HeadBias {
    const __nv_bfloat16* b[kHeadsPerLaunch];
};

// One CTA per root row, the row in registers (eight bf16 per 16-byte vector,
// at most kLnVec vectors per thread, so H <= 8 * 256 * kLnVec): mean and
// 1/std once, then y[i][row] = (x - mean) * rstd * w_i + b_i for each head i
// of the launch (two-pass statistics in fp32, as layer_norm computes them).
constexpr int kLnVec = 4;
__global__ void __launch_bounds__(256)
    layernorm_heads_kernel(const __nv_bfloat16* __restrict__ x, const __grid_constant__ HeadNorms hn, int32_t n,
                           int32_t B, int32_t dim, float eps, __nv_bfloat16* __restrict__ y) {
    __shared__ float red[32];
    const int nvec = dim / 8;
    const __nv_bfloat16* xr = x + (int64_t)blockIdx.x * dim;
    float v[kLnVec][8];
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < kLnVec; ++k) {
        const int vi = threadIdx.x + k * 256;
        if (vi < nvec) {
            const uint4 u = *reinterpret_cast<const uint4*>(xr + vi * 8);
            const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                v[k][j] = __bfloat162float(e[j]);
                s += v[k][j];
            }
        }
    }
    const float mean = block_sum<__nv_bfloat16>(s, red) / (float)dim;
    float q = 0.0f;
#pragma unroll
    for (int k = 0; k < kLnVec; ++k)
        if (threadIdx.x + k * 256 < nvec) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                v[k][j] -= mean;
                q += v[k][j] * v[k][j];
            }
        }
    const float r = rsqrtf(block_sum<__nv_bfloat16>(q, red) / (float)dim + eps);
    for (int h = 0; h < n; ++h) {
        __nv_bfloat16* yr = y + ((int64_t)h * B + blockIdx.x) * dim;
#pragma unroll
        for (int k = 0; k < kLnVec; ++k) {
            const int vi = threadIdx.x + k * 256;
            if (vi >= nvec) break;
            const uint4 uw = *reinterpret_cast<const uint4*>(hn.w[h] + vi * 8);
            const uint4 ub = *reinterpret_cast<const uint4*>(hn.b[h] + vi * 8);
            const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&uw);
            const __nv_bfloat16* be = reinterpret_cast<const __nv_bfloat16*>(&ub);
            uint4 res;
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(&res);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                o[j] = __float2bfloat16_rn(v[k][j] * r * __bfloat162float(we[j]) + __bfloat162float(be[j]));
            *reinterpret_cast<uint4*>(yr + vi * 8) = res;
        }
    }
}

// For head h of the launch, row r, columns c..c+3 (four per thread):
//   f = bf16(sum_s part[h][s][r][c] + bias_h[c]);  out[h][r][c] = bf16(x[r][c] + bf16(silu(f)))
// part [n][ksplit][B][H] fp32; the sums run in split order.
__global__ void fc_finish_kernel(const float* __restrict__ part, int32_t ksplit, const __grid_constant__ HeadBias hb,
                                 int32_t n, int32_t B, int32_t H, const __nv_bfloat16* __restrict__ x,
                                 __nv_bfloat16* __restrict__ out) {
    const int64_t bh = (int64_t)B * H, n_vec = (int64_t)n * bh / 4;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_vec; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = e * 4;
        const int h = (int)(o / bh);
        const int64_t rc = o - (int64_t)h * bh;
        const int32_t c = (int32_t)(rc % H);
        const float* ps = part + (int64_t)h * ksplit * bh + rc;
        float4 acc = *reinterpret_cast<const float4*>(ps);
        for (int sp = 1; sp < ksplit; ++sp) {
            const float4 v = *reinterpret_cast<const float4*>(ps + sp * bh);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        const __nv_bfloat16* bias = hb.b[h] + c;
        const float f[4] = {acc.x + __bfloat162float(bias[0]), acc.y + __bfloat162float(bias[1]),
                            acc.z + __bfloat162float(bias[2]), acc.w + __bfloat162float(bias[3])};
        const uint2 ux = *reinterpret_cast<const uint2*>(x + rc);
        const __nv_bfloat16* a = reinterpret_cast<const __nv_bfloat16*>(&ux);
        uint2 res;
        __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(&res);
#pragma unroll
        for (int j = 0; j < 4; ++j)
            d[j] = __float2bfloat16_rn(__bfloat162float(a[j]) +
                                       rnd<__nv_bfloat16>(silu(rnd<__nv_bfloat16>(f[j]))));
        *reinterpret_cast<uint2*>(out + o) = res;
    }
}

inline size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

}  // namespace prop
}  // namespace fg

extern "C" size_t fg_medusa_propose_workspace_size(int32_t B, int32_t H, int32_t V, int32_t n_heads, int32_t k) {
    if (B <= 0 || H <= 0 || V <= 0 || n_heads < 0) return 0;
    const size_t act = prop::align256((size_t)n_heads * B * H * sizeof(__nv_bfloat16));
    const size_t part = n_heads > 0 ? prop::align256((size_t)n_heads * lmh::part_split(H, H) * B * H * sizeof(float))
                                    : 0;
    const int32_t M = (1 + n_heads) * B;
    return act + part + (n_heads > 0 ? fg_lm_head_topk_workspace_size(M, V, B, k) : 0) + 256;
}

extern "C" fg_status fg_medusa_propose(void* x, int32_t dtype, int32_t B, int32_t H, const fg_medusa_head* heads,
                                       int32_t n_heads, float eps, const void* lm_head_w, int64_t w_ld, int32_t V,
                                       void* root_logits, int64_t logits_ld, int32_t k, int32_t* out_idx,
                                       float* out_val, float* out_max, float* out_lse, void* workspace,
                                       size_t workspace_bytes, void* stream) {
    if (B == 0) return FG_OK;
    if (dtype != FG_DTYPE_BF16) return FG_EUNSUPPORTED;
    if (!x || !lm_head_w || B < 0 || H <= 0 || V <= 0 || n_heads < 0 || (n_heads > 0 && !heads)) return FG_EINVAL;
    const int64_t M64 = (int64_t)(1 + n_heads) * B;
    if (M64 > lmh::kMaxRows || H % lmh::kKc || H > 8 * 256 * prop::kLnVec) return FG_ECAPACITY;
    if ((uintptr_t)x % 16) return FG_EINVAL;
    for (int i = 0; i < n_heads; ++i) {
        const fg_medusa_head& h = heads[i];
        if (!h.norm_w || !h.norm_b || !h.fc_w || !h.fc_b || ((uintptr_t)h.fc_w % 16) || ((uintptr_t)h.norm_w % 16) ||
            ((uintptr_t)h.norm_b % 16) || ((uintptr_t)h.fc_b % 8))
            return FG_EINVAL;
    }
    const int32_t M = (int32_t)M64;
    const size_t need = fg_medusa_propose_workspace_size(B, H, V, n_heads, k);
    if (n_heads > 0 && (!workspace || workspace_bytes < need || ((uintptr_t)workspace % 256))) return FG_ECAPACITY;
    cudaStream_t st = (cudaStream_t)stream;
    const __nv_bfloat16* hid = (const __nv_bfloat16*)x;
    const size_t act = prop::align256((size_t)n_heads * B * H * sizeof(__nv_bfloat16));
    const int ksplit = lmh::part_split(H, H);
    const size_t part_bytes = n_heads > 0 ? prop::align256((size_t)n_heads * ksplit * B * H * sizeof(float)) : 0;
    if (n_heads > 0) {
        __nv_bfloat16* ln = (__nv_bfloat16*)workspace;
        float* part = (float*)((uint8_t*)workspace + act);
        const int64_t bh = (int64_t)B * H;
        for (int h0 = 0; h0 < n_heads; h0 += prop::kHeadsPerLaunch) {
            const int n = n_heads - h0 < prop::kHeadsPerLaunch ? n_heads - h0 : prop::kHeadsPerLaunch;
            prop::HeadNorms hn{};
            for (int i = 0; i < n; ++i) {
                hn.w[i] = (const __nv_bfloat16*)heads[h0 + i].norm_w;
                hn.b[i] = (const __nv_bfloat16*)heads[h0 + i].norm_b;
            }
            prop::layernorm_heads_kernel<<<B, 256, 0, st>>>(hid, hn, n, B, H, eps, ln + h0 * bh);
            const fg_status s = launch_status();
            if (s != FG_OK) return s;
        }
        for (int i = 0; i < n_heads; ++i) {
            const fg_status s = lmh::run_partials(ln + i * bh, B, H, heads[i].fc_w, H, part + (int64_t)i * ksplit * bh,
                                                  stream);
            if (s != FG_OK) return s;
        }
        for (int h0 = 0; h0 < n_heads; h0 += prop::kHeadsPerLaunch) {
            const int n = n_heads - h0 < prop::kHeadsPerLaunch ? n_heads - h0 : prop::kHeadsPerLaunch;
            prop::HeadBias hb{};
            for (int i = 0; i < n; ++i) hb.b[i] = (const __nv_bfloat16*)heads[h0 + i].fc_b;
            const int64_t g = ((int64_t)n * bh / 4 + 255) / 256;
            prop::fc_finish_kernel<<<(int)(g < 148 * 8 ? g : 148 * 8), 256, 0, st>>>(
                part + (int64_t)h0 * ksplit * bh, ksplit, hb, n, B, H, hid, (__nv_bfloat16*)x + (1 + h0) * bh);
            const fg_status s = launch_status();
            if (s != FG_OK) return s;
        }
    }
    void* lws = n_heads > 0 ? (uint8_t*)workspace + act + part_bytes : nullptr;
    const size_t lws_bytes = n_heads > 0 ? workspace_bytes - act - part_bytes : 0;
    return fg_lm_head_topk(x, dtype, H, M, H, lm_head_w, w_ld, V, root_logits ? B : 0, root_logits, logits_ld, B, k,
                           out_idx, out_val, out_max, out_lse, lws, lws_bytes, stream);
}

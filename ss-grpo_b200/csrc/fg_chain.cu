// fg_chain.cu -- fg_chain_step: one level of a Chain-MEDUSA proposal (the
// ChainDraftCell on the chosen tokens, then the lm_head top-k of the new
// states) in one call.
//
// Per pass of at most 256 rows: one kernel gathers each row's parent state
// and token embedding and applies both LayerNorms; the state and token
// projections (H -> bottleneck) and the output projection (bottleneck -> H)
// run as the split-K partial-sum form of the lm_head kernel; two passes add
// the partial sums, one mixing (bf16(state_proj) + bf16(token_proj) -> SiLU)
// and one finishing (bias, sigmoid gate, residual); then fg_lm_head_topk.
// Rounding follows ChainDraftCell.forward (flashgrpo_b200/models/
// medusa_heads.py:154-160) in bf16: every torch op rounds its result.
#include "fg_common.cuh"

namespace fg {
namespace chain {

constexpr int kPassRows = 256;  // the lm_head kernel's row limit
constexpr int kLnVec = 4;       // 16-byte vectors per thread: H <= 8 * 256 * kLnVec

struct Cell {
    const __nv_bfloat16* sn_w;
    const __nv_bfloat16* sn_b;
    const __nv_bfloat16* tn_w;
    const __nv_bfloat16* tn_b;
    const __nv_bfloat16* out_b;
    const __nv_bfloat16* gate;
};

struct Rows {
    const int32_t* tokens;
    int32_t tok_ld, n_parent, fanout, n_child, V;
};

// Parent state row and token of chain row r; an out-of-range token records
// FG_EINVAL and reads embedding row 0.
__device__ __forceinline__ void row_source(const Rows& g, int32_t r, int32_t& srow, int32_t& tok) {
    const int32_t b = r / g.n_child, j = r - b * g.n_child;
    srow = b * g.n_parent + j / g.fanout;
    tok = g.tokens[(int64_t)b * g.tok_ld + j];
    if (tok < 0 || tok >= g.V) {
        atomicCAS(&g_fg_error_word, 0, FG_EINVAL);
        tok = 0;
    }
}

// y = (x - mean) * rstd * w + b of one row held in registers (256 threads).
__device__ __forceinline__ void ln_row(const __nv_bfloat16* __restrict__ xr, const __nv_bfloat16* __restrict__ w,
                                       const __nv_bfloat16* __restrict__ bb, int32_t dim, float eps,
                                       __nv_bfloat16* __restrict__ yr, float* red) {
    const int nvec = dim / 8;
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
#pragma unroll
    for (int k = 0; k < kLnVec; ++k) {
        const int vi = threadIdx.x + k * 256;
        if (vi >= nvec) break;
        const uint4 uw = *reinterpret_cast<const uint4*>(w + vi * 8);
        const uint4 ub = *reinterpret_cast<const uint4*>(bb + vi * 8);
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

// One CTA per row of the pass: ln_s[i] = LN_s(parent state), ln_t[i] = LN_t(embed[token]).
__global__ void __launch_bounds__(256)
    chain_norms_kernel(const __nv_bfloat16* __restrict__ state, const __grid_constant__ Rows g,
                       const __nv_bfloat16* __restrict__ embed, int64_t embed_ld, int32_t r0, int32_t H, float eps,
                       const __grid_constant__ Cell c, __nv_bfloat16* __restrict__ ln_s,
                       __nv_bfloat16* __restrict__ ln_t) {
    __shared__ float red[32];
    int32_t srow, tok;
    row_source(g, r0 + (int32_t)blockIdx.x, srow, tok);
    ln_row(state + (int64_t)srow * H, c.sn_w, c.sn_b, H, eps, ln_s + (int64_t)blockIdx.x * H, red);
    ln_row(embed + (int64_t)tok * embed_ld, c.tn_w, c.tn_b, H, eps, ln_t + (int64_t)blockIdx.x * H, red);
}

// act[i][c] = bf16(silu(bf16(bf16(sum_s ps[s][i][c]) + bf16(sum_s pt[s][i][c])))), four columns per thread.
__global__ void chain_mix_kernel(const float* __restrict__ ps, const float* __restrict__ pt, int32_t ksplit,
                                 int64_t n, __nv_bfloat16* __restrict__ act) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n / 4; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = e * 4;
        float4 a = *reinterpret_cast<const float4*>(ps + o);
        float4 b = *reinterpret_cast<const float4*>(pt + o);
        for (int s = 1; s < ksplit; ++s) {
            const float4 u = *reinterpret_cast<const float4*>(ps + s * n + o);
            const float4 w = *reinterpret_cast<const float4*>(pt + s * n + o);
            a.x += u.x;
            a.y += u.y;
            a.z += u.z;
            a.w += u.w;
            b.x += w.x;
            b.y += w.y;
            b.z += w.z;
            b.w += w.w;
        }
        const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
        uint2 res;
        __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(&res);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float mixed = rnd<__nv_bfloat16>(rnd<__nv_bfloat16>(av[j]) + rnd<__nv_bfloat16>(bv[j]));
            d[j] = __float2bfloat16_rn(silu(mixed));
        }
        *reinterpret_cast<uint2*>(act + o) = res;
    }
}

// out[r0 + i][c] = bf16(s + bf16(bf16(sigmoid(gate)) * bf16(sum_s po[s][i][c] + out_b[c]))), s the parent state.
__global__ void chain_out_kernel(const float* __restrict__ po, int32_t ksplit, const __nv_bfloat16* __restrict__ state,
                                 const __grid_constant__ Rows g, const __grid_constant__ Cell c, int32_t r0, int32_t m,
                                 int32_t H, __nv_bfloat16* __restrict__ out) {
    const int64_t n = (int64_t)m * H;
    const float gv = __bfloat162float(*c.gate);
    const float gate = rnd<__nv_bfloat16>(1.0f / (1.0f + expf(-gv)));
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n / 4; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = e * 4;
        const int32_t i = (int32_t)(o / H), col = (int32_t)(o - (int64_t)i * H);
        float4 a = *reinterpret_cast<const float4*>(po + o);
        for (int s = 1; s < ksplit; ++s) {
            const float4 u = *reinterpret_cast<const float4*>(po + s * n + o);
            a.x += u.x;
            a.y += u.y;
            a.z += u.z;
            a.w += u.w;
        }
        int32_t srow, tok;
        row_source(g, r0 + i, srow, tok);
        const uint2 us = *reinterpret_cast<const uint2*>(state + (int64_t)srow * H + col);
        const uint2 ub = *reinterpret_cast<const uint2*>(c.out_b + col);
        const __nv_bfloat16* sv = reinterpret_cast<const __nv_bfloat16*>(&us);
        const __nv_bfloat16* bv = reinterpret_cast<const __nv_bfloat16*>(&ub);
        const float av[4] = {a.x, a.y, a.z, a.w};
        uint2 res;
        __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(&res);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float delta = rnd<__nv_bfloat16>(av[j] + __bfloat162float(bv[j]));
            d[j] = __float2bfloat16_rn(__bfloat162float(sv[j]) + rnd<__nv_bfloat16>(gate * delta));
        }
        *reinterpret_cast<uint2*>(out + (int64_t)(r0 + i) * H + col) = res;
    }
}

inline size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

// Workspace layout for passes of up to m_max rows.
struct Layout {
    size_t ln_s, ln_t, ps, pt, act, po, lm, total;
};
inline Layout layout(int32_t m_max, int32_t H, int32_t bn, int32_t V, int32_t k) {
    const int s1 = lmh::part_split(bn, H), s2 = lmh::part_split(H, bn);
    Layout l;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off += align256(bytes);
        return at;
    };
    l.ln_s = take((size_t)m_max * H * 2);
    l.ln_t = take((size_t)m_max * H * 2);
    l.ps = take((size_t)s1 * m_max * bn * 4);
    l.pt = take((size_t)s1 * m_max * bn * 4);
    l.act = take((size_t)m_max * bn * 2);
    l.po = take((size_t)s2 * m_max * H * 4);
    l.lm = take(k > 0 ? fg_lm_head_topk_workspace_size(m_max, V, 0, k) : 0);
    l.total = off + 256;
    return l;
}

inline int elementwise_grid(int64_t n_vec) {
    const int64_t g = (n_vec + 255) / 256;
    return (int)(g < 148 * 8 ? (g > 0 ? g : 1) : 148 * 8);
}

}  // namespace chain
}  // namespace fg

extern "C" size_t fg_chain_step_workspace_size(int32_t M, int32_t H, int32_t bottleneck, int32_t V, int32_t k) {
    if (M <= 0 || H <= 0 || bottleneck <= 0 || V <= 0 || k < 0) return 0;
    return chain::layout(M < chain::kPassRows ? M : chain::kPassRows, H, bottleneck, V, k).total;
}

extern "C" fg_status fg_chain_step(const void* state, const int32_t* tokens, int32_t tok_ld, int32_t n_seq,
                                   int32_t n_parent, int32_t fanout, int32_t n_child, const void* embed,
                                   int64_t embed_ld, int32_t H, int32_t dtype, const fg_chain_cell* cell, float eps,
                                   void* state_out, const void* lm_head_w, int64_t w_ld, int32_t V, int32_t k,
                                   int32_t* out_idx, float* out_val, float* out_max, float* out_lse,
                                   void* workspace, size_t workspace_bytes, void* stream) {
    if (n_seq == 0 || n_child == 0) return FG_OK;
    if (dtype != FG_DTYPE_BF16) return FG_EUNSUPPORTED;
    if (!state || !tokens || !embed || !cell || !state_out || n_seq < 0 || n_child < 0 || n_parent <= 0 ||
        fanout <= 0 || tok_ld < n_child || (int64_t)n_parent * fanout < n_child || H <= 0 || V <= 0 || k < 0 ||
        embed_ld < H || embed_ld % 8)
        return FG_EINVAL;
    const int32_t bn = cell->bottleneck;
    if (H % 64 || bn <= 0 || bn % 64 || H > 8 * 256 * chain::kLnVec) return FG_ECAPACITY;
    if (k > 0 && (!lm_head_w || !out_idx || !out_val || !out_max)) return FG_EINVAL;
    if (k > FG_MAX_TOPK || k > V) return FG_ECAPACITY;
    const void* ptrs16[] = {state, embed, state_out, cell->state_norm_w, cell->state_norm_b, cell->token_norm_w,
                            cell->token_norm_b, cell->state_proj_w, cell->token_proj_w, cell->out_proj_w};
    for (const void* q : ptrs16)
        if (!q || ((uintptr_t)q % 16)) return FG_EINVAL;
    if (!cell->out_proj_b || ((uintptr_t)cell->out_proj_b % 8) || !cell->gate || ((uintptr_t)cell->gate % 2))
        return FG_EINVAL;
    const int64_t M64 = (int64_t)n_seq * n_child;
    if (M64 > 0x7fffffff) return FG_ECAPACITY;
    const int32_t M = (int32_t)M64;
    const int64_t n_state = (int64_t)n_seq * n_parent;
    {  // state_out must not overlap state (rows are contiguous, H elements)
        const uintptr_t s0 = (uintptr_t)state, s1 = s0 + (uintptr_t)(n_state * H * 2);
        const uintptr_t o0 = (uintptr_t)state_out, o1 = o0 + (uintptr_t)(M64 * H * 2);
        if (o0 < s1 && s0 < o1) return FG_EINVAL;
    }
    const int32_t m_max = M < chain::kPassRows ? M : chain::kPassRows;
    const chain::Layout L = chain::layout(m_max, H, bn, V, k);
    if (!workspace || workspace_bytes < L.total || ((uintptr_t)workspace % 256)) return FG_ECAPACITY;
    uint8_t* ws = (uint8_t*)workspace;
    __nv_bfloat16* ln_s = (__nv_bfloat16*)(ws + L.ln_s);
    __nv_bfloat16* ln_t = (__nv_bfloat16*)(ws + L.ln_t);
    float* ps = (float*)(ws + L.ps);
    float* pt = (float*)(ws + L.pt);
    __nv_bfloat16* act = (__nv_bfloat16*)(ws + L.act);
    float* po = (float*)(ws + L.po);
    const int s1 = lmh::part_split(bn, H), s2 = lmh::part_split(H, bn);
    chain::Cell c{(const __nv_bfloat16*)cell->state_norm_w, (const __nv_bfloat16*)cell->state_norm_b,
                  (const __nv_bfloat16*)cell->token_norm_w, (const __nv_bfloat16*)cell->token_norm_b,
                  (const __nv_bfloat16*)cell->out_proj_b,   (const __nv_bfloat16*)cell->gate};
    chain::Rows g{tokens, tok_ld, n_parent, fanout, n_child, V};
    cudaStream_t st = (cudaStream_t)stream;
    const __nv_bfloat16* sp = (const __nv_bfloat16*)state;
    __nv_bfloat16* out = (__nv_bfloat16*)state_out;
    for (int32_t r0 = 0; r0 < M; r0 += chain::kPassRows) {
        const int32_t m = M - r0 < chain::kPassRows ? M - r0 : chain::kPassRows;
        chain::chain_norms_kernel<<<m, 256, 0, st>>>(sp, g, (const __nv_bfloat16*)embed, embed_ld, r0, H, eps, c,
                                                     ln_s, ln_t);
        fg_status s = launch_status();
        if (s != FG_OK) return s;
        if ((s = lmh::run_partials(ln_s, m, H, cell->state_proj_w, bn, ps, stream)) != FG_OK) return s;
        if ((s = lmh::run_partials(ln_t, m, H, cell->token_proj_w, bn, pt, stream)) != FG_OK) return s;
        const int64_t n_mix = (int64_t)m * bn;
        chain::chain_mix_kernel<<<chain::elementwise_grid(n_mix / 4), 256, 0, st>>>(ps, pt, s1, n_mix, act);
        if ((s = launch_status()) != FG_OK) return s;
        if ((s = lmh::run_partials(act, m, bn, cell->out_proj_w, H, po, stream)) != FG_OK) return s;
        chain::chain_out_kernel<<<chain::elementwise_grid((int64_t)m * H / 4), 256, 0, st>>>(po, s2, sp, g, c, r0, m,
                                                                                             H, out);
        if ((s = launch_status()) != FG_OK) return s;
        if (k > 0) {
            s = fg_lm_head_topk(out + (int64_t)r0 * H, dtype, H, m, H, lm_head_w, w_ld, V, 0, nullptr, 0, 0, k,
                                out_idx + (int64_t)r0 * k, out_val + (int64_t)r0 * k, out_max + r0,
                                out_lse ? out_lse + r0 : nullptr, ws + L.lm, workspace_bytes - L.lm, stream);
            if (s != FG_OK) return s;
        }
    }
    return FG_OK;
}

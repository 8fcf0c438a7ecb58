// fg_attention.cu -- K3 host side: flash-decoding GQA attention of the tree
// queries, and the exact fp32 kernel.
//
// Replaces the HF eager/SDPA attention with the dense additive 4D mask that
// forward_tree runs (flashgrpo_b200/models/qwen_flashgrpo_wrapper.py:220-239,
// mask from flashgrpo_b200/decoding/tree_attention.py:6-67): prefix slots are
// visible to every node, tree slot j to node i iff bit j of anc_bits[i].
//
// bf16 path (head_dim 128): tc::attn_tc_kernel (fg_attention_tc.cu), grid
// (split, kv_head x row_group, row); KV heads with more than 128 query rows
// take tc::attn_tc_wide_kernel (fg_attention_tc2.cu, 256 rows per CTA).  A CTA owns the query rows of one KV head
// -- row r = node * G + g, up to 128 rows -- and streams its share of the
// row's KV slots [0, kv_len + n_nodes) through 4-D tensor maps over
// [B, Hkv, capacity, D] (128-slot x 64-dim boxes, 128-byte swizzle).  With
// several splits, each CTA writes (O, m, l) partials and the last CTA of a
// (row, head, group) merges them (a counter in the workspace that the merging
// CTA resets to zero).
// f32 path: one warp per query head, exact fp32 dot products (parity checks
// of the fp32 configuration).
#include <cstdio>

#include "fg_common.cuh"

// g_fg_error_word is defined in fg_abi.cu (same translation unit).

namespace fg {

constexpr int kD = 128;
constexpr int kMaxRows = 128;

// ------------------------------------------------------------------- f32
__global__ void tree_attn_f32_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                     const float* __restrict__ vc, int64_t sb, int64_t sh, int64_t ss,
                                     const int32_t* __restrict__ kv_len, const uint32_t* __restrict__ anc, int32_t N,
                                     int32_t Hq, int32_t Hkv, int32_t D, float scale, const int32_t* __restrict__ kv_rows,
                                     int32_t kv_batch, float* __restrict__ out) {
    const int node = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int G = Hq / Hkv;
    const int g = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (g >= G) return;
    const int hq = kvh * G + g;
    const float* qrow = q + (((int64_t)b * N + node) * Hq + hq) * D;
    float qv[4], acc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        qv[j] = d < D ? qrow[d] : 0.0f;
        acc[j] = 0.0f;
    }
    const int L = kv_len[b];
    const int T = L + N;
    float m = -INFINITY, l = 0.0f;
    const int32_t bk = max(cache_row(kv_rows, kv_batch, b), 0);  // an unmapped row reads row 0 (error recorded)
    const float* kb = kc + (int64_t)bk * sb + (int64_t)kvh * sh;
    const float* vb = vc + (int64_t)bk * sb + (int64_t)kvh * sh;
    for (int pos = 0; pos < T; ++pos) {
        if (pos >= L) {
            const int j = pos - L;
            if (!((anc[node * 4 + (j >> 5)] >> (j & 31)) & 1u)) continue;
        }
        float part = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int d = lane + 32 * j;
            if (d < D) part += qv[j] * kb[(int64_t)pos * ss + d];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        const float s = part * scale;
        const float mn = fmaxf(m, s);
        const float alpha = expf(m - mn);
        const float pw = expf(s - mn);
        l = l * alpha + pw;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int d = lane + 32 * j;
            acc[j] = acc[j] * alpha + (d < D ? pw * vb[(int64_t)pos * ss + d] : 0.0f);
        }
        m = mn;
    }
    float* orow = out + (((int64_t)b * N + node) * Hq + hq) * D;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int d = lane + 32 * j;
        if (d < D) orow[d] = l > 0.0f ? acc[j] / l : 0.0f;
    }
}

// ------------------------------------------------------------ host helpers
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// 4-D map over [B, Hkv, capacity, D] bf16 with 128-slot x 64-dim boxes, 128B swizzle.
static bool make_kv_map(CUtensorMap* map, void* base, int32_t B, int32_t Hkv, int32_t cap, int64_t sb, int64_t sh,
                        int64_t ss) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)cap, (cuuint64_t)Hkv, (cuuint64_t)B};
    const cuuint64_t strides[3] = {(cuuint64_t)ss * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
    const cuuint32_t box[4] = {64, (cuuint32_t)tc::kBlk, 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int auto_splits(int32_t items, int32_t max_kv_len, int32_t n_nodes) {
    const int chunks = (max_kv_len + n_nodes + tc::kBlk - 1) / tc::kBlk;
    const int slots = 148;  // one tensor-core CTA per SM (~194 KB of shared memory each)
    int s = slots / max(1, items);
    s = max(1, min(s, chunks / 2));
    return min(s, 64);
}

}  // namespace fg

using namespace fg;

// How a bf16 call runs: 129-256 query rows per KV head take the wide
// kernel (one 256-row group, a pair of 128-row sub-items in the workspace)
// when its grid fills the GPU without splits (at least kWideMinItems
// items), the rest the 128-row kernel; splits per item as requested or
// auto.  Measured: at 256 rows and >= 256 items the wide kernel is 3-22 %
// faster; with 64 items it needs 2 splits and is 55 % slower (the 7B shape
// with 16 rows per GPU), and with 512 rows its halved grid quantises worse
// onto the SMs (10-13 % slower).  Workspace: per sub-item and split the fp32 (O, m, l) partials,
// then one counter per item.
constexpr int kWideMinItems = 148;  // one CTA per SM

struct AttnPlan {
    bool wide;
    int groups;  // row groups per KV head (of 256 rows when wide, else 128)
    int items;   // B x Hkv x groups
    int subs;    // 128-row sub-items in the workspace
    int splits;
};

static AttnPlan plan_attention(int32_t B, int32_t n_nodes, int32_t n_q_heads, int32_t n_kv_heads, int32_t num_splits,
                               int32_t max_kv_len) {
    AttnPlan a;
    const int rows = n_nodes * (n_q_heads / n_kv_heads);
    a.wide = rows > kMaxRows && rows <= tc::kWideRows && B * n_kv_heads >= kWideMinItems;
    const int per = a.wide ? tc::kWideRows : kMaxRows;
    a.groups = (rows + per - 1) / per;
    a.items = B * n_kv_heads * a.groups;
    a.subs = a.wide ? 2 * a.items : a.items;
    a.splits = num_splits > 0 ? num_splits : auto_splits(a.items, max_kv_len, n_nodes);
    return a;
}

static size_t plan_workspace_bytes(const AttnPlan& a) {
    if (a.splits <= 1) return 0;
    return (size_t)a.subs * a.splits * (size_t)(kMaxRows * kD + 2 * kMaxRows) * sizeof(float) +
           (size_t)a.items * sizeof(int32_t);
}

extern "C" size_t fg_tree_attention_workspace_size(int32_t B, int32_t n_nodes, int32_t n_q_heads, int32_t n_kv_heads,
                                                   int32_t head_dim, int32_t num_splits, int32_t max_kv_len) {
    if (B <= 0 || n_nodes <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads || max_kv_len < 0 ||
        num_splits > tc::kMaxSplits)
        return 0;
    (void)head_dim;
    return plan_workspace_bytes(plan_attention(B, n_nodes, n_q_heads, n_kv_heads, num_splits, max_kv_len));
}

extern "C" fg_status fg_tree_attention(const void* q, int32_t dtype, const fg_kv_layer* kv, const int32_t* kv_len,
                                       const uint32_t* anc_bits, int32_t B, int32_t n_nodes, int32_t n_q_heads,
                                       int32_t n_kv_heads, int32_t head_dim, float scale, void* out, void* workspace,
                                       size_t workspace_bytes, int32_t num_splits, int32_t max_kv_len, void* stream) {
    if (B == 0) return FG_OK;
    if (!q || !kv || !kv->k || !kv->v || !kv_len || !anc_bits || !out || B < 0 || n_nodes <= 0 || n_kv_heads <= 0 ||
        n_q_heads % n_kv_heads)
        return FG_EINVAL;
    if (n_nodes > FG_MAX_TREE_NODES) return FG_ECAPACITY;
    if (num_splits > tc::kMaxSplits) return FG_EINVAL;
    if (kv->rows && kv->batch <= 0) return FG_EINVAL;
    const int32_t cache_b = kv->rows ? kv->batch : B;  // rows of the K/V tensors
    cudaStream_t st = (cudaStream_t)stream;
    if (dtype == FG_DTYPE_F32) {
        const int G = n_q_heads / n_kv_heads;
        if (head_dim > 128 || G > 32) return FG_ECAPACITY;
        dim3 grid(n_nodes, n_kv_heads, B);
        tree_attn_f32_kernel<<<grid, 32 * G, 0, st>>>((const float*)q, (const float*)kv->k, (const float*)kv->v,
                                                      kv->stride_b, kv->stride_h, kv->stride_s, kv_len, anc_bits,
                                                      n_nodes, n_q_heads, n_kv_heads, head_dim, scale, kv->rows,
                                                      kv->batch, (float*)out);
        return launch_status();
    }
    if (dtype != FG_DTYPE_BF16) return FG_EUNSUPPORTED;
    if (head_dim != kD) return FG_EUNSUPPORTED;
    if (((uintptr_t)kv->k % 16) || ((uintptr_t)kv->v % 16) || ((kv->stride_s * 2) % 16) || ((kv->stride_h * 2) % 16) ||
        ((kv->stride_b * 2) % 16) || ((uintptr_t)q % 16) || ((uintptr_t)out % 16))
        return FG_EINVAL;
    const int G = n_q_heads / n_kv_heads;
    tc::Params p;
    p.q = (const __nv_bfloat16*)q;
    p.out = (__nv_bfloat16*)out;
    p.kv_len = kv_len;
    p.anc = anc_bits;
    p.N = n_nodes;
    p.Hq = n_q_heads;
    p.Hkv = n_kv_heads;
    p.G = G;
    p.rows_total = n_nodes * G;
    const AttnPlan plan = plan_attention(B, n_nodes, n_q_heads, n_kv_heads, num_splits,
                                         max_kv_len > 0 ? max_kv_len : kv->capacity);
    p.groups = plan.groups;
    p.splits = plan.splits;
    // the kernel takes the row maximum of the raw scores and applies the scale
    // inside the exponent, which needs a positive scale
    if (!(scale > 0.0f)) return FG_EINVAL;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.ws_o = nullptr;
    p.ws_ml = nullptr;
    p.ws_cnt = nullptr;
    p.kv_rows = kv->rows;
    p.kv_batch = kv->batch;
    if (p.splits > 1) {
        const size_t need = plan_workspace_bytes(plan);
        if (!workspace || workspace_bytes < need || ((uintptr_t)workspace % 16)) return FG_ECAPACITY;
        p.ws_o = (float*)workspace;
        p.ws_ml = p.ws_o + (size_t)plan.subs * p.splits * kMaxRows * kD;
        p.ws_cnt = (int32_t*)(p.ws_ml + (size_t)plan.subs * p.splits * 2 * kMaxRows);
    }
    CUtensorMap mk, mv;
    if (!make_kv_map(&mk, kv->k, cache_b, n_kv_heads, kv->capacity, kv->stride_b, kv->stride_h, kv->stride_s) ||
        !make_kv_map(&mv, kv->v, cache_b, n_kv_heads, kv->capacity, kv->stride_b, kv->stride_h, kv->stride_s))
        return FG_EINVAL;
    static bool attr_set[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[plan.wide][dev]) {
        cudaError_t e = plan.wide ? cudaFuncSetAttribute(tc::attn_tc_wide_kernel,
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kWSmemBytes)
                                  : cudaFuncSetAttribute(tc::attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                         tc::kSmemBytes);
        if (e != cudaSuccess) {
            set_cuda_error(e);
            return FG_ECUDA;
        }
        if (dev >= 0 && dev < 64) attr_set[plan.wide][dev] = true;
    }
    // Programmatic launch: the CTAs may start (TMEM, barriers, prefix tile
    // loads) while the preceding kernel of the stream finishes; the kernel
    // waits for it (griddepcontrol.wait) before reading Q or tree slots.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.splits, n_kv_heads * p.groups, B);
    cfg.blockDim = dim3(tc::kThreads);
    cfg.dynamicSmemBytes = plan.wide ? tc::kWSmemBytes : tc::kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = plan.wide ? cudaLaunchKernelEx(&cfg, tc::attn_tc_wide_kernel, mk, mv, p)
                                    : cudaLaunchKernelEx(&cfg, tc::attn_tc_kernel, mk, mv, p);
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return FG_ECUDA;
    }
    return launch_status();
}

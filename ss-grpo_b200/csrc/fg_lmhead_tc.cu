// fg_lmhead_tc.cu -- K1: the tied lm_head projection of the proposal rows on
// the tensor cores, with the per-row top-k fused into the epilogue.
//
// Replaces, for bf16 policies, the concat-heads lm_head GEMM of
// _medusa_logits_for_last_hidden (flashgrpo_b200/decoding/
// flash_medusa_decoder.py:906-1005) followed by the per-head torch.topk of
// build_batch_trees (decoding/medusa_tree.py:767) and the confidence
// reductions (max, logsumexp) of flash_medusa_decoder.py:1021-1040.
//
// logits[r, v] = bf16( sum_k X[r, k] * W[v, k] ), X [M, H] (M <= 256 rows:
// the root row of every sequence, then each active head's projection), W the
// lm_head [V, H].  Rows [0, n_logit_rows) have their full bf16 logits written
// (the root sampler needs them); rows [topk_row0, M) get the top-k of their
// bf16 logits (value descending, index ascending), the row maximum and,
// optionally, the logsumexp -- exactly what fg_row_topk returns on the
// written logits -- without the logits ever reaching HBM.
//
// One persistent CTA per SM owns a contiguous vocab range (balanced in units
// of 16 columns).  Tiles are 256 vocab columns x all rows (two M=128 blocks):
//   warp 0       TMA: per 64-wide k chunk, the W tile (256 x 64, or 16-row
//                boxes for a narrow last tile) and the X chunk, 128-byte
//                swizzle, into a ring as deep as shared memory allows (4
//                stages for 192 rows) (no L2 prefetch of W: prefetching
//                chunks twelve ahead measured 12 % slower, 170 vs 150 us);
//   warp 1       allocates 512 TMEM columns (M block b -> columns
//                [256 b, 256 b + 256)); one thread issues tcgen05.mma
//                D[b] (+)= X[b rows] * W_tile^T, commits stages and tiles;
//   warps 4-11   epilogue: warp w takes TMEM lanes 32 (w % 4).. and one column
//                half of every tile in both M blocks (two rows per thread):
//                tcgen05.ld, round to bf16, write logits rows, keep sorted
//                top-k lists (branch-free insertion) and an online (max, sum
//                exp); per (CTA, half) partials go to the workspace and a
//                second kernel merges them per row.
// X is re-read from L2 for every tile (0.75 bytes per byte of W); W streams
// from HBM once.  Every mbarrier wait is bounded (about one second).
#include "fg_common.cuh"

namespace fg {
namespace lmh {

using tc::bar_drain;
using tc::bar_expect;
using tc::bar_init;
using tc::bar_arrive;
using tc::bar_wait;
using tc::fence_after;
using tc::fence_before;
using tc::sa;
using tc::sdesc;
using tc::tld32;
using tc::umma;
using tc::umma_commit;

constexpr int kN = 256;                   // vocab columns per tile
constexpr int kKc = 64;                   // k elements per stage (128-byte rows)
constexpr int kMaxStages = 6;            // ring depth is chosen at launch from the X box size
constexpr int kThreads = 384;
constexpr int kMaxRows = 256;
constexpr int kWBytes = kN * 128;         // 32 KB
constexpr int kOffStage = 1024;          // barriers in the first 1 KB, stages after
constexpr int kSmemBytes = 232448;        // the sm_100 per-CTA maximum
constexpr uint32_t kTmemCols = 512;
constexpr int kUnit = 16;                 // vocab split granularity (MMA N step)

struct Params {
    int32_t M, H, V, n_units, nk;
    int32_t stages, stage_bytes;  // ring depth, bytes per stage: [X box | W tile], 1 KB multiples
    int32_t x_area;               // bytes of the X box rounded up to 1 KB (W starts there)
    int32_t xrows;          // rows of the X box (multiple of 8, >= M)
    int32_t n_logit_rows;   // rows [0, n) write logits
    __nv_bfloat16* logits;
    int64_t logits_ld;
    int32_t logits_vec;     // rows 16-byte aligned: vector stores
    int32_t topk_row0, k, want_lse;
    int32_t* part_idx;      // [M - topk_row0][2 nctas][k] (per CTA, per column half)
    float* part_val;
    float* part_m;          // [M - topk_row0][2 nctas]
    float* part_s;
    int32_t ksplit;         // partial-sum form: CTAs per column group, each over nk / ksplit k chunks
    float* part;            // partial-sum form: [ksplit][M][V] fp32 sums, unrounded
};

struct Bars {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t acc_full;
    uint64_t acc_free;
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
};

// L2 eviction policies: X (small, re-read for every tile) is kept, the W
// stream (read once) goes first.
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* b,
                                       uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
        "{%2, %3}], [%4], %5;" ::"r"(sa(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(sa(b)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ bool better(float av, int32_t ai, float bv, int32_t bi) {
    return av > bv || (av == bv && ai < bi);
}

// vocab range [u0 * 16, u1 * 16) of CTA c: units split as evenly as possible
__device__ __forceinline__ void cta_range(int n_units, int c, int nctas, int& u0, int& u1) {
    const int base = n_units / nctas, extra = n_units % nctas;
    u0 = c * base + min(c, extra);
    u1 = u0 + base + (c < extra ? 1 : 0);
}

// kPart: the partial-sum form for narrow GEMMs (the MEDUSA head fc layers,
// V = H): CTA c takes column group c / ksplit (at most 128 columns) and k
// range (c % ksplit) of the nk chunks, and stores its fp32 sums unrounded
// into part[c % ksplit]; a separate pass adds them up.  No logits, no top-k.
template <int K, bool kPart = false>
__global__ void __launch_bounds__(kThreads, 1) lmhead_topk_kernel(const __grid_constant__ CUtensorMap tmW256,
                                                                  const __grid_constant__ CUtensorMap tmW16,
                                                                  const __grid_constant__ CUtensorMap tmX, Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem);
    const int kStages = p.stages;
    volatile int* abort_flag = &bars->abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int u0, u1, kc0 = 0, kc1 = p.nk;
    const int ks = kPart ? (int)blockIdx.x % p.ksplit : 0;
    if constexpr (kPart) {
        cta_range(p.n_units, blockIdx.x / p.ksplit, gridDim.x / p.ksplit, u0, u1);
        kc0 = ks * p.nk / p.ksplit;
        kc1 = (ks + 1) * p.nk / p.ksplit;
    } else {
        cta_range(p.n_units, blockIdx.x, gridDim.x, u0, u1);
    }
    const int v_begin = u0 * kUnit, v_end = min(u1 * kUnit, p.V);
    const int n_tiles = (u1 - u0 + (kN / kUnit) - 1) / (kN / kUnit);
    const int nmb = p.M > 128 ? 2 : 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            bar_init(&bars->full[s], 1);
            bar_init(&bars->empty[s], 1);
        }
        bar_init(&bars->acc_full, 1);
        bar_init(&bars->acc_free, 8);
        bar_init(&bars->drain, 1);
        bars->abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(&bars->tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA
        if (lane == 0) {
            const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
            int it = 0, issued = 0;
            bool ok = true;
            for (int t = 0; t < n_tiles && ok; ++t) {
                const int v0 = v_begin + t * kN;
                const int w = min(kN, u1 * kUnit - v0);  // multiple of 16
                const uint32_t bytes = (uint32_t)w * 128u + (uint32_t)p.xrows * 128u;
                for (int kc = kc0; kc < kc1; ++kc, ++it) {
                    const int s = it % kStages;
                    if (it >= kStages && !(ok = bar_wait(&bars->empty[s], ((it / kStages) - 1) & 1, abort_flag)))
                        break;
                    uint8_t* st = smem + kOffStage + s * p.stage_bytes;
                    bar_expect(&bars->full[s], bytes);
                    uint8_t* sw = st + p.x_area;
                    if (w == kN) {
                        tma_2d(sw, &tmW256, kc * kKc, v0, &bars->full[s], pol_w);
                    } else {
                        for (int j = 0; j < w / kUnit; ++j)
                            tma_2d(sw + j * kUnit * 128, &tmW16, kc * kKc, v0 + j * kUnit, &bars->full[s], pol_w);
                    }
                    tma_2d(st, &tmX, kc * kKc, 0, &bars->full[s], pol_x);
                    issued = it + 1;
                }
            }
            for (int j = max(0, issued - kStages); j < issued; ++j)
                bar_drain(&bars->full[j % kStages], (j / kStages) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int t = 0; t < n_tiles && ok; ++t) {
                const int v0 = v_begin + t * kN;
                const int w = min(kN, u1 * kUnit - v0);
                const uint32_t idesc = tc::idesc_bf16(w, false);
                if (t > 0 && !(ok = bar_wait(&bars->acc_free, (t - 1) & 1, abort_flag))) break;
                fence_after();
                for (int kc = kc0; kc < kc1; ++kc, ++it) {
                    const int s = it % kStages;
                    if (!(ok = bar_wait(&bars->full[s], (it / kStages) & 1, abort_flag))) break;
                    fence_after();
                    // M block 1 reads X rows 128..255 = stage bytes [16 KB, 32 KB):
                    // rows past the X box fall on this stage's W bytes (garbage
                    // rows >= M, never read back), always inside the stage
                    const uint32_t x_addr = sa(smem + kOffStage + s * p.stage_bytes);
                    const uint32_t w_addr = x_addr + (uint32_t)p.x_area;
                    for (int b = 0; b < nmb; ++b) {
#pragma unroll
                        for (int kk = 0; kk < kKc / 16; ++kk) {
                            const uint64_t da = sdesc(x_addr + b * (128 * 128) + kk * 32, 16, 1024);
                            const uint64_t db = sdesc(w_addr + kk * 32, 16, 1024);
                            umma(tmem + (uint32_t)(b * kN), da, db, idesc, (kc > kc0 || kk > 0) ? 1u : 0u);
                        }
                    }
                    umma_commit(&bars->empty[s]);
                }
                if (ok) umma_commit(&bars->acc_full);
            }
            umma_commit(&bars->drain);
            bar_drain(&bars->drain, 0);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------- epilogue
        // Warp w reads TMEM lanes 32 (w % 4) .. + 31 and takes column half
        // h = (w - 4) / 4 of every tile, in both M blocks: each thread owns
        // two rows (32 (w % 4) + lane and that + 128), so every warp gets the
        // same share whichever rows write logits or keep a top-k.
        constexpr unsigned kFull = 0xffffffffu;
        const int q4 = warp & 3, h = (warp - 4) >> 2;
        const uint32_t lane_addr = tmem + ((uint32_t)(q4 * 32) << 16);
        // per row: the running list (value desc, index asc) in kL independent
        // sub-lists (element j of a chunk goes to list j % kL and each list
        // still sees increasing indices), merged at the end
        constexpr int kL = K <= 4 ? 4 : 1;
        float lv[2][kL][K];
        int32_t li[2][kL][K];
        float m[2] = {-INFINITY, -INFINITY}, sx[2] = {0.0f, 0.0f};
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int l = 0; l < kL; ++l)
#pragma unroll
                for (int j = 0; j < K; ++j) {
                    lv[b][l][j] = -INFINITY;
                    li[b][l][j] = 0x7fffffff;
                }
        bool ok = true;
        for (int t = 0; t < n_tiles; ++t) {
            const int v0 = v_begin + t * kN;
            const int w = min(kN, u1 * kUnit - v0);
            if (!__all_sync(kFull, bar_wait(&bars->acc_full, t & 1, abort_flag))) {
                ok = false;
                break;
            }
            fence_after();
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                if (b >= nmb) break;
                const int row = b * 128 + q4 * 32 + lane;
                const bool valid = row < p.M;
                const bool write = valid && row < p.n_logit_rows;
                const bool topk = valid && row >= p.topk_row0;
                for (int c = h * (kN / 2); c < min(w, (h + 1) * (kN / 2)); c += 32) {
                    float x[32];
                    tld32(lane_addr + (uint32_t)(b * kN + c), x);
                    const int vb = v0 + c;
                    if constexpr (kPart) {
                        if (valid) {
                            float* dst = p.part + ((int64_t)ks * p.M + row) * p.V + vb;
                            if (vb + 32 <= v_end) {  // V is a multiple of 64 here: 16-byte aligned
#pragma unroll
                                for (int qq = 0; qq < 8; ++qq)
                                    *reinterpret_cast<float4*>(dst + 4 * qq) =
                                        make_float4(x[4 * qq], x[4 * qq + 1], x[4 * qq + 2], x[4 * qq + 3]);
                            } else {
#pragma unroll
                                for (int j = 0; j < 32; ++j)
                                    if (vb + j < v_end) dst[j] = x[j];
                            }
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) x[j] = __bfloat162float(__float2bfloat16_rn(x[j]));
                        if (write) {
                            __nv_bfloat16* dst = p.logits + (int64_t)row * p.logits_ld + vb;
                            if (p.logits_vec && vb + 32 <= v_end) {
#pragma unroll
                                for (int qq = 0; qq < 4; ++qq) {
                                    uint4 u;
                                    u.x = tc::pack2(x[8 * qq + 0], x[8 * qq + 1]);
                                    u.y = tc::pack2(x[8 * qq + 2], x[8 * qq + 3]);
                                    u.z = tc::pack2(x[8 * qq + 4], x[8 * qq + 5]);
                                    u.w = tc::pack2(x[8 * qq + 6], x[8 * qq + 7]);
                                    *reinterpret_cast<uint4*>(dst + 8 * qq) = u;
                                }
                            } else {
#pragma unroll
                                for (int j = 0; j < 32; ++j)
                                    if (vb + j < v_end) dst[j] = __float2bfloat16_rn(x[j]);
                            }
                        }
                        if (topk) {
                            const int n_ok = min(32, v_end - vb);
#pragma unroll
                            for (int j = 0; j < 32; ++j) x[j] = j < n_ok ? x[j] : -INFINITY;
                            if (p.want_lse) {
                                float cm[8];
#pragma unroll
                                for (int qq = 0; qq < 8; ++qq)
                                    cm[qq] = fmaxf(fmaxf(x[qq], x[qq + 8]), fmaxf(x[qq + 16], x[qq + 24]));
                                const float cmax = fmaxf(fmaxf(fmaxf(cm[0], cm[1]), fmaxf(cm[2], cm[3])),
                                                         fmaxf(fmaxf(cm[4], cm[5]), fmaxf(cm[6], cm[7])));
                                if (cmax != -INFINITY) {
                                    // online (max, sum exp) one chunk at a time
                                    const float mn = fmaxf(m[b], cmax);
                                    float e = 0.0f;
#pragma unroll
                                    for (int j = 0; j < 32; ++j) e += expf(x[j] - mn);  // masked: exp(-inf) = 0
                                    sx[b] = (m[b] == -INFINITY ? 0.0f : sx[b] * expf(m[b] - mn)) + e;
                                    m[b] = mn;
                                }
                            }
                            // branch-free insertion: an element passes only strictly
                            // smaller values (equal values keep the smaller index)
#pragma unroll
                            for (int j = 0; j < 32; ++j) {
                                const int l = j & (kL - 1);
                                float cv = x[j];
                                int32_t ci = vb + j;
#pragma unroll
                                for (int qq = 0; qq < K; ++qq) {
                                    const bool gt = cv > lv[b][l][qq];
                                    const float nv = gt ? cv : lv[b][l][qq];
                                    const int32_t ni = gt ? ci : li[b][l][qq];
                                    cv = gt ? lv[b][l][qq] : cv;
                                    ci = gt ? li[b][l][qq] : ci;
                                    lv[b][l][qq] = nv;
                                    li[b][l][qq] = ni;
                                }
                            }
                        }
                    }
                }
            }
            fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&bars->acc_free);
        }
        // merge the sub-lists of each row (full comparator) and publish
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            const int row = b * 128 + q4 * 32 + lane;
            if (b >= nmb || !ok || *abort_flag || row >= p.M || row < p.topk_row0) continue;
            float tv[K];
            int32_t ti[K];
#pragma unroll
            for (int j = 0; j < K; ++j) {
                tv[j] = lv[b][0][j];
                ti[j] = li[b][0][j];
            }
#pragma unroll
            for (int l = 1; l < kL; ++l) {
#pragma unroll
                for (int e = 0; e < K; ++e) {
                    float cv = lv[b][l][e];
                    int32_t ci = li[b][l][e];
#pragma unroll
                    for (int qq = 0; qq < K; ++qq) {
                        const bool gt = better(cv, ci, tv[qq], ti[qq]);
                        const float nv = gt ? cv : tv[qq];
                        const int32_t ni = gt ? ci : ti[qq];
                        cv = gt ? tv[qq] : cv;
                        ci = gt ? ti[qq] : ci;
                        tv[qq] = nv;
                        ti[qq] = ni;
                    }
                }
            }
            // partial list number (CTA, column half)
            const int64_t pr = (int64_t)(row - p.topk_row0) * (2 * gridDim.x) + 2 * blockIdx.x + h;
#pragma unroll
            for (int j = 0; j < K; ++j) {
                if (j < p.k) {
                    p.part_idx[pr * p.k + j] = ti[j];
                    p.part_val[pr * p.k + j] = tv[j];
                }
            }
            p.part_m[pr] = p.want_lse ? m[b] : tv[0];
            p.part_s[pr] = p.want_lse ? sx[b] : 0.0f;
        }
        fence_before();
    }
    __syncthreads();
    fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// Per row: k rounds of "best head among the per-CTA lists" (the lists are
// sorted, so the global top-k is a k-way merge), and the logsumexp from the
// per-CTA (max, sum exp) pairs.
__global__ void __launch_bounds__(256) lmhead_merge_kernel(const int32_t* __restrict__ part_idx,
                                                           const float* __restrict__ part_val,
                                                           const float* __restrict__ part_m,
                                                           const float* __restrict__ part_s, int32_t nctas, int32_t k,
                                                           int32_t want_lse, int32_t* __restrict__ out_idx,
                                                           float* __restrict__ out_val, float* __restrict__ out_max,
                                                           float* __restrict__ out_lse) {
    __shared__ float redv[8];
    __shared__ int32_t redi[8];
    __shared__ int32_t redt[8];
    __shared__ float reds[8];
    __shared__ int32_t winner;
    const int tid = threadIdx.x, r = blockIdx.x;
    const int32_t* pi = part_idx + (int64_t)r * nctas * k;
    const float* pv = part_val + (int64_t)r * nctas * k;
    // thread tid owns the lists of CTAs tid, tid + 256, ...; heads advance on wins
    int head[4] = {0, 0, 0, 0};
    const int n_own = (nctas - tid + 255) / 256;
    for (int rr = 0; rr < k; ++rr) {
        float bv = -INFINITY;
        int32_t bi = 0x7fffffff;
        int bl = -1;
        for (int q = 0; q < n_own && q < 4; ++q) {
            const int c = tid + q * 256;
            if (head[q] < k) {
                const float v = pv[c * k + head[q]];
                const int32_t i = pi[c * k + head[q]];
                if (better(v, i, bv, bi) || bl < 0) {
                    bv = v;
                    bi = i;
                    bl = q;
                }
            }
        }
        int bt = bl < 0 ? 0x7fffffff : tid * 4 + bl;
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
            float wv = tid < 8 ? redv[tid] : -INFINITY;
            int32_t wi = tid < 8 ? redi[tid] : 0x7fffffff;
            int wt = tid < 8 ? redt[tid] : 0x7fffffff;
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
                out_idx[(int64_t)r * k + rr] = (wi == 0x7fffffff) ? 0 : wi;
                out_val[(int64_t)r * k + rr] = wv;
                if (rr == 0) out_max[r] = wv;
            }
        }
        __syncthreads();
        if (winner != 0x7fffffff && (winner >> 2) == tid) ++head[winner & 3];
        __syncthreads();
    }
    if (want_lse && out_lse != nullptr) {
        float gm = -INFINITY;
        for (int c = tid; c < nctas; c += 256) gm = fmaxf(gm, part_m[(int64_t)r * nctas + c]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
        if ((tid & 31) == 0) redv[tid >> 5] = gm;
        __syncthreads();
        gm = redv[0];
        for (int w = 1; w < 8; ++w) gm = fmaxf(gm, redv[w]);
        float ls = 0.0f;
        for (int c = tid; c < nctas; c += 256) {
            const float mc = part_m[(int64_t)r * nctas + c];
            if (mc != -INFINITY) ls += part_s[(int64_t)r * nctas + c] * expf(mc - gm);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
        if ((tid & 31) == 0) reds[tid >> 5] = ls;
        __syncthreads();
        if (tid == 0) {
            float tot = 0.0f;
            for (int w = 0; w < 8; ++w) tot += reds[w];
            out_lse[r] = __bfloat162float(__float2bfloat16_rn(gm + logf(tot)));
        }
    }
}

static bool make_map_2d(CUtensorMap* map, const void* base, int64_t inner, int64_t rows, int64_t ld_elems,
                        uint32_t box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld_elems * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kKc, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int sm_count() {
    static int n[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (n[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        n[dev] = v;
    }
    return n[dev];
}

static int grid_for(int32_t V) {
    const int units = (V + kUnit - 1) / kUnit;
    return units < sm_count() ? units : sm_count();
}

}  // namespace lmh
}  // namespace fg

using namespace fg;

extern "C" size_t fg_lm_head_topk_workspace_size(int32_t M, int32_t V, int32_t topk_row0, int32_t k) {
    if (M <= 0 || V <= 0 || k <= 0 || topk_row0 < 0 || topk_row0 >= M) return 0;
    // two partial lists per CTA (its two column halves)
    const size_t rows = (size_t)(M - topk_row0), nlists = 2 * (size_t)lmh::grid_for(V);
    return rows * nlists * ((size_t)k * 8 + 8) + 256;
}

namespace fg {
namespace lmh {

static fg_status run(const void* x, int32_t dtype, int64_t x_ld, int32_t M, int32_t H, const void* w, int64_t w_ld,
                     int32_t V, int32_t n_logit_rows, void* logits, int64_t logits_ld, int32_t topk_row0, int32_t k,
                     int32_t* out_idx, float* out_val, float* out_max, float* out_lse, void* workspace,
                     size_t workspace_bytes, void* stream) {
    if (M == 0) return FG_OK;
    if (dtype != FG_DTYPE_BF16) return FG_EUNSUPPORTED;
    if (!x || !w || M < 0 || V <= 0 || H <= 0 || n_logit_rows < 0 || n_logit_rows > M || topk_row0 < 0 ||
        topk_row0 > M)
        return FG_EINVAL;
    if (M > lmh::kMaxRows || H % lmh::kKc) return FG_ECAPACITY;
    if (((uintptr_t)x % 16) || ((uintptr_t)w % 16) || (x_ld % 8) || (w_ld % 8) || x_ld < H || w_ld < H)
        return FG_EINVAL;
    if (n_logit_rows > 0 && (!logits || ((uintptr_t)logits % 2) || logits_ld < V)) return FG_EINVAL;
    const bool has_topk = topk_row0 < M;
    if (has_topk) {
        if (!out_idx || !out_val || !out_max) return FG_EINVAL;
        if (k <= 0 || k > FG_MAX_TOPK || k > V) return FG_ECAPACITY;
    }
    const int nctas = lmh::grid_for(V);
    lmh::Params p;
    p.M = M;
    p.H = H;
    p.V = V;
    p.n_units = (V + lmh::kUnit - 1) / lmh::kUnit;
    p.nk = H / lmh::kKc;
    p.xrows = (M + 7) & ~7;
    p.x_area = (p.xrows * 128 + 1023) & ~1023;
    p.stage_bytes = p.x_area + lmh::kWBytes;  // >= 32 KB + 1 KB: the M block 1 window fits
    p.stages = (lmh::kSmemBytes - 1024 - lmh::kOffStage) / p.stage_bytes;
    if (p.stages > lmh::kMaxStages) p.stages = lmh::kMaxStages;
    p.n_logit_rows = n_logit_rows;
    p.logits = (__nv_bfloat16*)logits;
    p.logits_ld = logits_ld;
    p.logits_vec = (((uintptr_t)logits % 16) == 0 && (logits_ld % 8) == 0) ? 1 : 0;
    p.topk_row0 = has_topk ? topk_row0 : M;
    p.k = has_topk ? k : 1;
    p.want_lse = out_lse != nullptr ? 1 : 0;
    p.part_idx = nullptr;
    p.part_val = p.part_m = p.part_s = nullptr;
    p.ksplit = 1;
    p.part = nullptr;
    if (has_topk) {
        const size_t need = fg_lm_head_topk_workspace_size(M, V, topk_row0, k);
        if (!workspace || workspace_bytes < need || ((uintptr_t)workspace % 16)) return FG_ECAPACITY;
        const size_t rows = (size_t)(M - topk_row0) * 2 * nctas;
        p.part_idx = (int32_t*)workspace;
        p.part_val = (float*)(p.part_idx + rows * k);
        p.part_m = p.part_val + rows * k;
        p.part_s = p.part_m + rows;
    }
    CUtensorMap m256, m16, mx;
    if (!lmh::make_map_2d(&m256, w, H, V, w_ld, lmh::kN) || !lmh::make_map_2d(&m16, w, H, V, w_ld, lmh::kUnit) ||
        !lmh::make_map_2d(&mx, x, H, M, x_ld, (uint32_t)p.xrows))
        return FG_EINVAL;
    static bool attr_set[64][5] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int kk = !has_topk ? 0 : k <= 1 ? 0 : k <= 2 ? 1 : k <= 4 ? 2 : k <= 8 ? 3 : 4;
    cudaStream_t st = (cudaStream_t)stream;
    auto launch = [&](auto kern) -> fg_status {
        if (dev < 0 || dev >= 64 || !attr_set[dev][kk]) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, lmh::kSmemBytes);
            if (e != cudaSuccess) {
                set_cuda_error(e);
                return FG_ECUDA;
            }
            if (dev >= 0 && dev < 64) attr_set[dev][kk] = true;
        }
        kern<<<nctas, lmh::kThreads, lmh::kSmemBytes, st>>>(m256, m16, mx, p);
        return launch_status();
    };
    fg_status s;
    switch (kk) {
        case 0: s = launch(lmh::lmhead_topk_kernel<1>); break;
        case 1: s = launch(lmh::lmhead_topk_kernel<2>); break;
        case 2: s = launch(lmh::lmhead_topk_kernel<4>); break;
        case 3: s = launch(lmh::lmhead_topk_kernel<8>); break;
        default: s = launch(lmh::lmhead_topk_kernel<16>); break;
    }
    if (s != FG_OK || !has_topk) return s;
    lmh::lmhead_merge_kernel<<<M - topk_row0, 256, 0, st>>>(p.part_idx, p.part_val, p.part_m, p.part_s, 2 * nctas, k,
                                                           p.want_lse, out_idx, out_val, out_max, out_lse);
    return launch_status();
}

// Partial-sum form: column groups of at most 8 units (128 columns), and as
// many k ranges per group as fill the SMs once (at most nk).
static int part_groups(int32_t V) { return ((V + kUnit - 1) / kUnit + 7) / 8; }
static int part_split(int32_t V, int32_t H) {
    const int g = part_groups(V), nk = H / kKc;
    const int s = sm_count() / g;
    return s < 1 ? 1 : s > nk ? nk : s;
}

// part[ks][r][v] = the sum over k chunks [ks nk / S, (ks + 1) nk / S) of
// x[r, k] w[v, k] (fp32, unrounded) for x [M, H], w [V, H] bf16 (row strides
// H), S = part_split(V, H); part holds S * M * V floats, 16-byte aligned.
static fg_status run_partials(const void* x, int32_t M, int32_t H, const void* w, int32_t V, float* part,
                              void* stream) {
    if (!x || !w || !part || M <= 0 || M > kMaxRows || H % kKc || V % 64 || ((uintptr_t)x % 16) ||
        ((uintptr_t)w % 16) || ((uintptr_t)part % 16))
        return FG_EINVAL;
    Params p{};
    p.M = M;
    p.H = H;
    p.V = V;
    p.n_units = (V + kUnit - 1) / kUnit;
    p.nk = H / kKc;
    p.xrows = (M + 7) & ~7;
    p.x_area = (p.xrows * 128 + 1023) & ~1023;
    p.stage_bytes = p.x_area + kWBytes;
    p.stages = (kSmemBytes - 1024 - kOffStage) / p.stage_bytes;
    if (p.stages > kMaxStages) p.stages = kMaxStages;
    p.topk_row0 = M;
    p.k = 1;
    p.ksplit = part_split(V, H);
    p.part = part;
    CUtensorMap m256, m16, mx;
    if (!make_map_2d(&m256, w, H, V, H, kN) || !make_map_2d(&m16, w, H, V, H, kUnit) ||
        !make_map_2d(&mx, x, H, M, H, (uint32_t)p.xrows))
        return FG_EINVAL;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    auto kern = lmhead_topk_kernel<1, true>;
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) {
            set_cuda_error(e);
            return FG_ECUDA;
        }
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    kern<<<part_groups(V) * p.ksplit, kThreads, kSmemBytes, (cudaStream_t)stream>>>(m256, m16, mx, p);
    return launch_status();
}

}  // namespace lmh
}  // namespace fg

extern "C" fg_status fg_lm_head_topk(const void* x, int32_t dtype, int64_t x_ld, int32_t M, int32_t H, const void* w,
                                     int64_t w_ld, int32_t V, int32_t n_logit_rows, void* logits, int64_t logits_ld,
                                     int32_t topk_row0, int32_t k, int32_t* out_idx, float* out_val, float* out_max,
                                     float* out_lse, void* workspace, size_t workspace_bytes, void* stream) {
    return lmh::run(x, dtype, x_ld, M, H, w, w_ld, V, n_logit_rows, logits, logits_ld, topk_row0, k, out_idx, out_val,
                    out_max, out_lse, workspace, workspace_bytes, stream);
}

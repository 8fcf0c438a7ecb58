// fg_gemm_tc.cu -- the dense projections of the verify forward on the tensor
// cores: D = X W^T with the consumer of D fused into the epilogue.
//
//   X [M, K] bf16 (tokens x hidden), W [N, K] bf16 (nn.Linear layout), fp32
//   accumulation in TMEM, one of three epilogues:
//     FG_EPI_STORE   out = bf16(D + bias)                 (QKV with bias,
//                                                          the lm_head rows)
//     FG_EPI_RESID   out = bf16(resid + D + bias)         (O and down
//                                                          projections with
//                                                          the residual add;
//                                                          resid may be out)
//     FG_EPI_SWIGLU  out = bf16(bf16(silu(bf16(g))) * bf16(u)), g / u the
//                    rows j and N + j of W               (gate/up + SwiGLU)
//   Each rounding is the one the reference's torch ops apply (addmm rounds
//   acc + bias [+ resid] once; the MLP rounds gate, up, silu and the product).
//
// Tiles: 128 tokens x bn outputs on one SM (bn a multiple of 16, <= 256;
// SwiGLU stacks the bn gate rows on the bn up rows, MMA N = 2 bn <= 256), or
// 256 tokens on a pair of SMs (below), 64-wide k chunks through a ring of
// shared-memory slots -- two chunks per slot when K has an even number of
// chunks, each operand of a slot one TMA box through a (64 k, row, chunk)
// tensor map, since an SM takes in more bytes per second with fewer, larger
// TMA instructions.  The epilogue and the ring depth are template
// parameters, so the kernels carry no per-element mode branches.  Work units
// are (output tile, k range): with split-K the units write fp32 partial
// tiles to a workspace and a second kernel adds them in k order and applies
// the epilogue, so results do not depend on which CTA finishes first.
// Persistent grid, units ordered weight-tile-major so the token tiles
// sharing a weight tile run together and the weights stream from HBM about
// once:
//   warp 0     TMA producer (X box 128 rows x 64 k x cps chunks, W box bn rows
//              x 64 k x cps chunks, 128-byte swizzle);
//   warp 1     allocates 512 TMEM columns (two accumulators, 256 apart); one
//              thread issues tcgen05.mma, commits stages and tiles;
//   warps 4-11 epilogue: warp w reads TMEM lanes 32 (w % 4) .. (one token row
//              per thread) and half (w - 4) / 4 of the tile's outputs; the
//              accumulator is released as soon as it is read, so the
//              epilogue of one unit overlaps the MMAs of the next.
// Programmatic dependent launch: the weight boxes of the first stages are
// requested before griddepcontrol.wait (weights are not written by the
// preceding kernels), X, bias and resid only after it; the CTA lets its
// dependents launch once its own wait has returned.  Every mbarrier wait is
// bounded (about one second) and records FG_ETIMEOUT.
#include "fg_common.cuh"

namespace fg {
namespace gemm {

using tc::bar_arrive;
using tc::bar_drain;
using tc::bar_expect;
using tc::bar_init;
using tc::bar_wait;
using tc::fence_after;
using tc::fence_before;
using tc::sa;
using tc::sdesc;
using tc::tld32;
using tc::umma;
using tc::umma_commit;

constexpr int kBM = 128;          // tokens per tile and CTA (MMA M of one SM)
constexpr int kKc = 64;           // k elements per stage (128-byte rows)
constexpr int kMaxStages = 8;
constexpr int kStages1 = 4;       // default ring depth of the 1-SM tile (4, 6 or 8 compiled)
constexpr int kStagesPair = 6;    // ring depth of the SM-pair tile
constexpr int kThreads = 384;
constexpr int kABytes = kBM * 128;  // 16 KB
constexpr int kOffStage = 1024;     // barriers in the first 1 KB
constexpr int kSmemMax = 227 * 1024;
constexpr uint32_t kTmemCols = 512;

struct Params {
    int32_t M, N, K;
    int32_t bn;        // outputs per tile
    int32_t nb;        // W rows per tile = MMA N (bn, or 2 bn for SwiGLU)
    int32_t n_mt, n_nt, splits, nk, units, stage_bytes;
    int32_t cps;       // 64-wide k chunks per ring stage (1, or 2 when nk is even)
    const __nv_bfloat16* bias;   // [N] or null
    const __nv_bfloat16* resid;  // FG_EPI_RESID: [M, ld_resid]
    int64_t ld_resid;
    __nv_bfloat16* out;
    int64_t ld_out;
    float* ws;                   // split-K partials [split][M][N] (SwiGLU [split][M][2N])
};

struct Bars {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
};

__device__ __forceinline__ void decode(const Params& p, int u, int& nt, int& ks, int& mt) {
    const int per_nt = p.splits * p.n_mt;
    nt = u / per_nt;
    const int r = u - nt * per_nt;
    ks = r / p.n_mt;
    mt = r - ks * p.n_mt;
}

// The k range [kc0, kc1) of split ks, in whole stages of cps chunks.
__device__ __forceinline__ void k_range(const Params& p, int ks, int& kc0, int& kc1) {
    const int np = p.nk / p.cps;
    kc0 = p.cps * (ks * np / p.splits);
    kc1 = p.cps * ((ks + 1) * np / p.splits);
}

// One stage's boxes through the k-chunked maps: coordinates (0, row, chunk)
// or, for the stacked gate/up weights, (0, row, half, chunk).  A box spans
// cps chunks, so a stage is one instruction per operand.
__device__ __forceinline__ void tma_3d(void* dst, const CUtensorMap* map, int row, int kc, uint64_t* b, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
        "{%2, %3, %4}], [%5], %6;" ::"r"(sa(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(row), "r"(kc), "r"(sa(b)), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void tma_4d(void* dst, const CUtensorMap* map, int row, int kc, uint64_t* b, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
        "{%2, %3, %4, %5}], [%6], %7;" ::"r"(sa(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(row), "r"(0), "r"(kc), "r"(sa(b)), "l"(pol)
        : "memory");
}

__device__ __forceinline__ float bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
// x * sigmoid(x) with the fast exponential and division intrinsics, as
// fg_silu_mul evaluates it (the result is rounded to bf16)
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// 8 bf16 held in a 16-byte vector, as floats
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __bfloat1622float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

// The bias and residual inputs of one 32-column chunk of a row, loaded ahead
// of the accumulator they are added to.  The loads of a chunk are issued
// together (and before the tile's MMAs finish): added one 8-wide group at a
// time, each load would wait behind the previous group's store, which may
// alias it (the residual add runs in place).
struct EpiIn {
    uint4 b[4];
    uint4 r[4];
};

template <int EPI>
__device__ __forceinline__ void epi_load(const Params& p, int row, int col0, int n, EpiIn& in) {
    if constexpr (EPI == FG_EPI_SWIGLU) return;
    if (p.splits != 1 || row >= p.M) return;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        if (8 * q < n && col0 + 8 * q < p.N) {
            if (p.bias) in.b[q] = *reinterpret_cast<const uint4*>(p.bias + col0 + 8 * q);
            if constexpr (EPI == FG_EPI_RESID)
                in.r[q] = *reinterpret_cast<const uint4*>(p.resid + (int64_t)row * p.ld_resid + col0 + 8 * q);
        }
    }
}

// The epilogue of 8 consecutive outputs [col, col + 8) of one row, from the
// fp32 accumulators g (and u for SwiGLU) and the preloaded bias / residual
// vectors, stored as one 16-byte vector.
template <int EPI>
__device__ __forceinline__ void finish8_in(const Params& p, int row, int col, const float* g, const float* u,
                                           const uint4& bq, const uint4& rq) {
    float o[8];
    if constexpr (EPI == FG_EPI_SWIGLU) {
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = bf(silu_f(bf(g[e]))) * bf(u[e]);
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = g[e];
        if (p.bias) {
            float b[8];
            unpack8(bq, b);
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] += b[e];
        }
        if constexpr (EPI == FG_EPI_RESID) {
            float r[8];
            unpack8(rq, r);
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] += r[e];
        }
    }
    uint4 v;
    v.x = tc::pack2(o[0], o[1]);
    v.y = tc::pack2(o[2], o[3]);
    v.z = tc::pack2(o[4], o[5]);
    v.w = tc::pack2(o[6], o[7]);
    *reinterpret_cast<uint4*>(p.out + (int64_t)row * p.ld_out + col) = v;
}

// finish8_in with its inputs loaded here (the split-K reduce, one group per thread)
template <int EPI>
__device__ __forceinline__ void finish8(const Params& p, int row, int col, const float* g, const float* u) {
    uint4 bq = make_uint4(0, 0, 0, 0), rq = make_uint4(0, 0, 0, 0);
    if constexpr (EPI != FG_EPI_SWIGLU) {
        if (p.bias) bq = *reinterpret_cast<const uint4*>(p.bias + col);
        if constexpr (EPI == FG_EPI_RESID) rq = *reinterpret_cast<const uint4*>(p.resid + (int64_t)row * p.ld_resid + col);
    }
    finish8_in<EPI>(p, row, col, g, u, bq, rq);
}

// One 32-column chunk of a warp's outputs after the TMEM reads: the epilogue
// of its 8-wide groups (one k range), or its fp32 partials (split-K).
template <int EPI>
__device__ __forceinline__ void emit32(const Params& p, int row, int col0, int n, int ks, const float* g,
                                       const float* u, const EpiIn& in) {
    if (row >= p.M) return;
    if (p.splits == 1) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (8 * q >= n || col0 + 8 * q >= p.N) break;
            finish8_in<EPI>(p, row, col0 + 8 * q, g + 8 * q, u + 8 * q, in.b[q], in.r[q]);
        }
    } else {
        const int64_t nw = EPI == FG_EPI_SWIGLU ? 2 * (int64_t)p.N : p.N;
        float* part = p.ws + ((int64_t)ks * p.M + row) * nw + col0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if (4 * q >= n || col0 + 4 * q >= p.N) break;
            __stcg(reinterpret_cast<float4*>(part + 4 * q),
                   make_float4(g[4 * q], g[4 * q + 1], g[4 * q + 2], g[4 * q + 3]));
            if constexpr (EPI == FG_EPI_SWIGLU)
                __stcg(reinterpret_cast<float4*>(part + p.N + 4 * q),
                       make_float4(u[4 * q], u[4 * q + 1], u[4 * q + 2], u[4 * q + 3]));
        }
    }
}

template <int EPI, int STAGES>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmX,
                                                           const __grid_constant__ CUtensorMap tmW, Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem);
    volatile int* abort_flag = &bars->abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int my_units = p.units > (int)blockIdx.x ? (p.units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int cps = p.cps;
    const uint32_t stage_tx = (uint32_t)p.stage_bytes;

    // W boxes of a stage: the tile's rows for cps chunks (SwiGLU: its gate
    // rows then its up rows per chunk, through the 4-D map)
    auto load_w = [&](uint8_t* st, int nt, int kc, uint64_t* bar, uint64_t pol) {
        if constexpr (EPI == FG_EPI_SWIGLU)
            tma_4d(st + cps * kABytes, &tmW, nt * p.bn, kc, bar, pol);
        else
            tma_3d(st + cps * kABytes, &tmW, nt * p.bn, kc, bar, pol);
    };
    // the first stages of this CTA's first unit: weights before the grid dependency wait
    int pre = 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            bar_init(&bars->full[s], 1);
            bar_init(&bars->empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            bar_init(&bars->acc_full[a], 1);
            bar_init(&bars->acc_empty[a], 8);
        }
        bar_init(&bars->drain, 1);
        bars->abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (my_units > 0) {
            int nt, ks, mt;
            decode(p, blockIdx.x, nt, ks, mt);
            int kc0, kc1;
            k_range(p, ks, kc0, kc1);
            pre = min(STAGES, (kc1 - kc0) / cps);
            const uint64_t pol_w = lmh::policy_evict_first();
            for (int j = 0; j < pre; ++j) {
                bar_expect(&bars->full[j], stage_tx);
                load_w(smem + kOffStage + j * p.stage_bytes, nt, kc0 + j * cps, &bars->full[j], pol_w);
            }
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(&bars->tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // X, bias and resid come from the preceding kernels
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA
        if (lane == 0) {
            const uint64_t pol_w = lmh::policy_evict_first(), pol_x = lmh::policy_evict_last();
            int it = 0, issued = 0;
            bool ok = true;
            for (int i = 0; i < my_units && ok; ++i) {
                int nt, ks, mt;
                decode(p, (int)blockIdx.x + i * (int)gridDim.x, nt, ks, mt);
                int kc0, kc1;
                k_range(p, ks, kc0, kc1);
                for (int kc = kc0; kc < kc1; kc += cps, ++it) {
                    const int s = it % STAGES;
                    if (it >= STAGES && !(ok = bar_wait(&bars->empty[s], ((it / STAGES) - 1) & 1, abort_flag)))
                        break;
                    uint8_t* st = smem + kOffStage + s * p.stage_bytes;
                    if (it >= pre) {
                        bar_expect(&bars->full[s], stage_tx);
                        load_w(st, nt, kc, &bars->full[s], pol_w);
                    }
                    tma_3d(st, &tmX, mt * kBM, kc, &bars->full[s], pol_x);
                    issued = it + 1;
                }
            }
            for (int j = max(0, issued - STAGES); j < issued; ++j)
                bar_drain(&bars->full[j % STAGES], (j / STAGES) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_bf16(p.nb, false);
            int it = 0;
            bool ok = true;
            for (int i = 0; i < my_units && ok; ++i) {
                int nt, ks, mt;
                decode(p, (int)blockIdx.x + i * (int)gridDim.x, nt, ks, mt);
                int kc0, kc1;
                k_range(p, ks, kc0, kc1);
                const int a = i & 1;
                if (i >= 2 && !(ok = bar_wait(&bars->acc_empty[a], ((i >> 1) - 1) & 1, abort_flag))) break;
                fence_after();
                for (int kc = kc0; kc < kc1; kc += cps, ++it) {
                    const int s = it % STAGES;
                    if (!(ok = bar_wait(&bars->full[s], (it / STAGES) & 1, abort_flag))) break;
                    fence_after();
                    const uint32_t a_base = sa(smem + kOffStage + s * p.stage_bytes);
                    const uint32_t b_base = a_base + (uint32_t)(cps * kABytes);
                    for (int c = 0; c < cps; ++c) {
                        const uint32_t a_addr = a_base + (uint32_t)(c * kABytes);
                        const uint32_t b_addr = b_base + (uint32_t)(c * p.nb * 128);
#pragma unroll
                        for (int kk = 0; kk < kKc / 16; ++kk)
                            umma(tmem + (uint32_t)(a * 256), sdesc(a_addr + kk * 32, 16, 1024),
                                 sdesc(b_addr + kk * 32, 16, 1024), idesc, (kc > kc0 || c > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(&bars->empty[s]);
                }
                if (ok) umma_commit(&bars->acc_full[a]);
            }
            umma_commit(&bars->drain);
            bar_drain(&bars->drain, 0);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------- epilogue
        // warp w: TMEM lanes 32 (w % 4) .. (one token row per thread) and
        // outputs [grp span, (grp + 1) span) of the tile
        const int q4 = warp & 3, grp = (warp - 4) >> 2;
        const uint32_t lane_addr = tmem + ((uint32_t)(q4 * 32) << 16);
        const int span = p.bn / 2, o0 = grp * span;
        for (int i = 0; i < my_units; ++i) {
            const int a = i & 1;
            int nt, ks, mt;
            decode(p, (int)blockIdx.x + i * (int)gridDim.x, nt, ks, mt);
            const int row = mt * kBM + q4 * 32 + lane;
            const int col0 = nt * p.bn + o0;
            // the first chunk's bias / residual load while the MMAs run
            EpiIn cur;
            epi_load<EPI>(p, row, col0, min(32, span), cur);
            if (!__all_sync(0xffffffffu, bar_wait(&bars->acc_full[a], (i >> 1) & 1, abort_flag))) break;
            fence_after();
            const uint32_t acc = lane_addr + (uint32_t)(a * 256);
            // 32-column TMEM reads (warp-uniform); columns past this warp's
            // range stay inside the accumulator and are dropped
#pragma unroll 1
            for (int c = 0; c < span; c += 32) {
                EpiIn nxt;
                if (c + 32 < span) epi_load<EPI>(p, row, col0 + c + 32, min(32, span - c - 32), nxt);
                float g[32], u[32];
                tld32(acc + (uint32_t)(o0 + c), g);
                if constexpr (EPI == FG_EPI_SWIGLU) tld32(acc + (uint32_t)(p.bn + o0 + c), u);
                emit32<EPI>(p, row, col0 + c, min(32, span - c), ks, g, u, cur);
                cur = nxt;
            }
            fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&bars->acc_empty[a]);
        }
        fence_before();
    }
    __syncthreads();
    fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// ------------------------------------------------------------ 2-SM tiles
// The same projection with 256-token tiles on a pair of SMs (a cluster of
// two CTAs, tcgen05 cta_group::2): each CTA loads its own 128 token rows and
// half of the tile's weight rows; the even CTA of the pair issues one M = 256
// MMA per 16-wide k step that reads both CTAs' shared memory and writes each
// CTA's 128 rows to that CTA's TMEM.  Per k chunk a CTA thus moves half the
// weight bytes of a 1-SM tile of the same width.  Protocol:
//   * both CTAs initialise their barriers, then a cluster barrier; warp 1 of
//     each CTA allocates the same 512 TMEM columns (cta_group::2);
//   * every TMA load (no multicast) completes its bytes on the even CTA's
//     full barrier of the stage, whose producer alone expects the bytes of
//     both CTAs; each CTA's producer reuses a stage after its own empty
//     barrier, which the even CTA's MMA commit signals in both CTAs;
//   * the MMA commit of a unit signals acc_full in both CTAs; the epilogue
//     warps of both CTAs release the accumulator on the even CTA's acc_empty
//     (16 arrivals);
//   * at the end the MMA thread waits for its last MMAs, a cluster barrier
//     keeps the odd CTA's shared memory and TMEM alive until then, and both
//     warps 1 free the TMEM.
// SwiGLU: the even CTA holds the bn gate rows, the odd CTA the bn up rows, so
// gate j and up j land in TMEM columns j and bn + j as in the 1-SM tile.
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same shared variable in the even CTA of the pair
__device__ __forceinline__ uint32_t at_rank0(const void* p) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(sa(p)));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// A stage's box through a k-chunked map, completing on the even CTA's barrier
__device__ __forceinline__ void tma_3d_pair(void* dst, const CUtensorMap* map, int row, int kc, uint32_t mbar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(sa(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(row), "r"(kc), "r"(mbar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void umma_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
// arrive on this barrier offset in both CTAs of the pair when the MMAs issued so far complete
__device__ __forceinline__ void umma_commit_pair(uint64_t* b) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            sa(b)),
        "h"((uint16_t)3)
        : "memory");
}
__device__ __forceinline__ void umma_commit_pair_local(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(b))
                 : "memory");
}
__device__ __forceinline__ void arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

template <int EPI, int STAGES>
__global__ void __launch_bounds__(kThreads, 1) gemm_pair_kernel(const __grid_constant__ CUtensorMap tmX,
                                                                const __grid_constant__ CUtensorMap tmW, Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem);
    volatile int* abort_flag = &bars->abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int cid = (int)blockIdx.x >> 1, ncl = (int)gridDim.x >> 1;
    const int my_units = p.units > cid ? (p.units - 1 - cid) / ncl + 1 : 0;
    const int bh = p.nb / 2;  // weight rows this CTA loads per chunk
    const int cps = p.cps;
    const uint32_t pair_tx = 2u * (uint32_t)p.stage_bytes;
    constexpr int kTile = 2 * kBM;  // tokens per tile
    auto w_row = [&](int nt) {
        return EPI == FG_EPI_SWIGLU ? (int)rank * p.N + nt * p.bn : nt * p.bn + (int)rank * bh;
    };

    int pre = 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            bar_init(&bars->full[s], 1);
            bar_init(&bars->empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            bar_init(&bars->acc_full[a], 1);
            bar_init(&bars->acc_empty[a], 16);
        }
        bar_init(&bars->drain, 1);
        bars->abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(&bars->tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before any load signals the even CTA's
    fence_after();
    const uint32_t tmem = bars->tmem_base;
    // weights of this pair's first stages before the grid dependency wait
    if (threadIdx.x == 0 && my_units > 0) {
        int nt, ks, mt;
        decode(p, cid, nt, ks, mt);
        int kc0, kc1;
        k_range(p, ks, kc0, kc1);
        pre = min(STAGES, (kc1 - kc0) / cps);
        const uint64_t pol_w = lmh::policy_evict_first();
        for (int j = 0; j < pre; ++j) {
            uint8_t* st = smem + kOffStage + j * p.stage_bytes;
            if (rank == 0) bar_expect(&bars->full[j], pair_tx);
            tma_3d_pair(st + cps * kABytes, &tmW, w_row(nt), kc0 + j * cps, at_rank0(&bars->full[j]), pol_w);
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == 0) {
        // ------------------------------------------------------------ TMA
        if (lane == 0) {
            const uint64_t pol_w = lmh::policy_evict_first(), pol_x = lmh::policy_evict_last();
            int it = 0, issued = 0;
            bool ok = true;
            for (int i = 0; i < my_units && ok; ++i) {
                int nt, ks, mt;
                decode(p, cid + i * ncl, nt, ks, mt);
                int kc0, kc1;
                k_range(p, ks, kc0, kc1);
                for (int kc = kc0; kc < kc1; kc += cps, ++it) {
                    const int s = it % STAGES;
                    if (it >= STAGES && !(ok = bar_wait(&bars->empty[s], ((it / STAGES) - 1) & 1, abort_flag)))
                        break;
                    uint8_t* st = smem + kOffStage + s * p.stage_bytes;
                    const uint32_t full0 = at_rank0(&bars->full[s]);
                    if (it >= pre) {
                        if (rank == 0) bar_expect(&bars->full[s], pair_tx);
                        tma_3d_pair(st + cps * kABytes, &tmW, w_row(nt), kc, full0, pol_w);
                    }
                    tma_3d_pair(st, &tmX, mt * kTile + (int)rank * kBM, kc, full0, pol_x);
                    issued = it + 1;
                }
            }
            // the even CTA's full barriers count both CTAs' bytes: its producer
            // waits for the last stages to land before the pair may finish
            if (rank == 0)
                for (int j = max(0, issued - STAGES); j < issued; ++j)
                    bar_drain(&bars->full[j % STAGES], (j / STAGES) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA
        if (lane == 0 && rank == 0) {
            const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.nb >> 3) << 17) |
                                   ((uint32_t)(kTile >> 4) << 24);
            int it = 0;
            bool ok = true;
            for (int i = 0; i < my_units && ok; ++i) {
                int nt, ks, mt;
                decode(p, cid + i * ncl, nt, ks, mt);
                int kc0, kc1;
                k_range(p, ks, kc0, kc1);
                const int a = i & 1;
                if (i >= 2 && !(ok = bar_wait(&bars->acc_empty[a], ((i >> 1) - 1) & 1, abort_flag))) break;
                fence_after();
                for (int kc = kc0; kc < kc1; kc += cps, ++it) {
                    const int s = it % STAGES;
                    if (!(ok = bar_wait(&bars->full[s], (it / STAGES) & 1, abort_flag))) break;
                    fence_after();
                    const uint32_t a_base = sa(smem + kOffStage + s * p.stage_bytes);
                    const uint32_t b_base = a_base + (uint32_t)(cps * kABytes);
                    for (int c = 0; c < cps; ++c) {
                        const uint32_t a_addr = a_base + (uint32_t)(c * kABytes);
                        const uint32_t b_addr = b_base + (uint32_t)(c * bh * 128);
#pragma unroll
                        for (int kk = 0; kk < kKc / 16; ++kk)
                            umma_pair(tmem + (uint32_t)(a * 256), sdesc(a_addr + kk * 32, 16, 1024),
                                      sdesc(b_addr + kk * 32, 16, 1024), idesc,
                                      (kc > kc0 || c > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit_pair(&bars->empty[s]);
                }
                if (ok) umma_commit_pair(&bars->acc_full[a]);
            }
            umma_commit_pair_local(&bars->drain);
            bar_drain(&bars->drain, 0);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------- epilogue
        const int q4 = warp & 3, grp = (warp - 4) >> 2;
        const uint32_t lane_addr = tmem + ((uint32_t)(q4 * 32) << 16);
        const int span = p.bn / 2, o0 = grp * span;
        const uint32_t empty0 = at_rank0(&bars->acc_empty[0]), empty1 = at_rank0(&bars->acc_empty[1]);
        for (int i = 0; i < my_units; ++i) {
            const int a = i & 1;
            int nt, ks, mt;
            decode(p, cid + i * ncl, nt, ks, mt);
            const int row = mt * kTile + (int)rank * kBM + q4 * 32 + lane;
            const int col0 = nt * p.bn + o0;
            EpiIn cur;
            epi_load<EPI>(p, row, col0, min(32, span), cur);
            if (!__all_sync(0xffffffffu, bar_wait(&bars->acc_full[a], (i >> 1) & 1, abort_flag))) break;
            fence_after();
            const uint32_t acc = lane_addr + (uint32_t)(a * 256);
#pragma unroll 1
            for (int c = 0; c < span; c += 32) {
                EpiIn nxt;
                if (c + 32 < span) epi_load<EPI>(p, row, col0 + c + 32, min(32, span - c - 32), nxt);
                float g[32], u[32];
                tld32(acc + (uint32_t)(o0 + c), g);
                if constexpr (EPI == FG_EPI_SWIGLU) tld32(acc + (uint32_t)(p.bn + o0 + c), u);
                emit32<EPI>(p, row, col0 + c, min(32, span - c), ks, g, u, cur);
                cur = nxt;
            }
            fence_before();
            __syncwarp();
            if (lane == 0) arrive_cluster(a ? empty1 : empty0);
        }
        fence_before();
    }
    __syncthreads();
    // the even CTA's MMAs have completed (its MMA thread drained them) and both
    // epilogues are done before either CTA frees TMEM or leaves
    cluster_sync();
    fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// out = epilogue(sum of the split-K partials in k order): one thread per 8
// consecutive outputs, the slots' float4 loads independent of each other.
template <int EPI>
__global__ void __launch_bounds__(256) linear_reduce_kernel(Params p) {
    pdl_wait_then_release();
    const int n8 = p.N / 8;
    const int64_t nw = EPI == FG_EPI_SWIGLU ? 2 * (int64_t)p.N : p.N;
    const int64_t total = (int64_t)p.M * n8;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(e / n8), col = (int)(e - (int64_t)row * n8) * 8;
        float g[8], u[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) g[k] = u[k] = 0.0f;
        const float* src = p.ws + (int64_t)row * nw + col;
#pragma unroll 2
        for (int s2 = 0; s2 < p.splits; ++s2) {
            const float* q = src + (int64_t)s2 * p.M * nw;
            const float4 x0 = __ldcg(reinterpret_cast<const float4*>(q));
            const float4 x1 = __ldcg(reinterpret_cast<const float4*>(q + 4));
            g[0] += x0.x; g[1] += x0.y; g[2] += x0.z; g[3] += x0.w;
            g[4] += x1.x; g[5] += x1.y; g[6] += x1.z; g[7] += x1.w;
            if constexpr (EPI == FG_EPI_SWIGLU) {
                const float4 y0 = __ldcg(reinterpret_cast<const float4*>(q + p.N));
                const float4 y1 = __ldcg(reinterpret_cast<const float4*>(q + p.N + 4));
                u[0] += y0.x; u[1] += y0.y; u[2] += y0.z; u[3] += y0.w;
                u[4] += y1.x; u[5] += y1.y; u[6] += y1.z; u[7] += y1.w;
            }
        }
        finish8<EPI>(p, row, col, g, u);
    }
}

// A tile shape is usable when every 32-column TMEM read of the epilogue
// stays inside its 256-column accumulator slot.  pair: the 2-SM tile, whose
// CTAs each load half of the nb weight rows.
static bool tile_ok(bool pair, int bn, int epi) {
    if (bn <= 0 || bn % 16) return false;
    const int nb = epi == FG_EPI_SWIGLU ? 2 * bn : bn;
    if (nb > 256) return false;
    if (pair && (nb / 2) % 8) return false;
    const int span = bn / 2, o0 = bn / 2;
    return o0 + (span + 31) / 32 * 32 + (epi == FG_EPI_SWIGLU ? bn : 0) <= 256;
}

static int stage_bytes(bool pair, int nb) { return kABytes + (pair ? nb / 2 : nb) * 128; }

static int fit_stages(bool pair, int nb) {
    return min(kMaxStages, (kSmemMax - 1024 - kOffStage) / stage_bytes(pair, nb));
}

// Tile shape for a problem: (tokens per tile 128 on one SM / 256 on an SM
// pair, outputs, k ranges) with the least estimated time.  Per 64-wide k
// chunk an SM moves stage_bytes from L2 (~45 bytes per clock) and issues
// 2 nb MMA clocks; a unit adds ~1500 clocks of fill and epilogue tail; split-K
// adds the partials' round trip.
static void choose_tile(int32_t M, int32_t N, int32_t K, int32_t epi, int sms, int max_splits, int32_t& bm_out,
                        int32_t& bn_out, int32_t& s_out) {
    const int nk = K / kKc;
    double best = 0.0;
    bn_out = 0;
    bm_out = kBM;
    s_out = 1;
    for (int pair = 0; pair <= 1; ++pair) {
        const int bm = pair ? 2 * kBM : kBM;
        const int n_mt = (M + bm - 1) / bm;
        const int slots = pair ? sms / 2 : sms;
        for (int bn = 256; bn >= 16; bn -= 16) {
            if (!tile_ok(pair, bn, epi) || (epi == FG_EPI_SWIGLU && N % bn)) continue;
            const int nb = epi == FG_EPI_SWIGLU ? 2 * bn : bn;
            const int n_nt = (N + bn - 1) / bn;
            for (int sp = 1; sp <= max_splits; ++sp) {
                if (sp > 1 && nk / sp < 4) break;
                const long units = (long)n_mt * n_nt * sp;
                const long waves = (units + slots - 1) / slots;
                const double chunk = fmax(2.0 * nb, stage_bytes(pair, nb) / 45.0);
                double cost = (double)waves * ((double)nk / sp * chunk + 1500.0);
                if (sp > 1) cost += (double)sp * M * N * 8.0 / (45.0 * sms) + 2000.0;
                if (bn_out == 0 || cost < best) {
                    best = cost;
                    bn_out = bn;
                    bm_out = bm;
                    s_out = sp;
                }
            }
        }
    }
}

static size_t ws_bytes(int32_t M, int32_t N, int32_t epi, int32_t splits) {
    if (splits <= 1) return 0;
    return (size_t)splits * M * (epi == FG_EPI_SWIGLU ? 2 * (size_t)N : (size_t)N) * sizeof(float);
}

// bm / bn / splits / stages <= 0: chosen here
static void resolve(int32_t M, int32_t N, int32_t K, int32_t epi, int32_t& bm, int32_t& bn, int32_t& splits,
                    int32_t& stages) {
    if (bm <= 0 || bn <= 0 || splits <= 0) {
        int32_t bm2, b2, s2;
        choose_tile(M, N, K, epi, lmh::sm_count(), splits > 0 ? splits : 8, bm2, b2, s2);
        if (bm <= 0) bm = bm2;
        if (bn <= 0) bn = b2;
        if (splits <= 0) splits = s2;
    }
    if (stages <= 0) stages = bm == 2 * kBM ? kStagesPair : kStages1;
}

// Launches one instantiation, raising its dynamic shared memory limit on
// the first launch of that instantiation on each device.
template <void (*KERNEL)(CUtensorMap, CUtensorMap, Params)>
static cudaError_t launch_tile(cudaLaunchConfig_t& cfg, const CUtensorMap& mx, const CUtensorMap& mw,
                               const Params& p) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(KERNEL, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    return cudaLaunchKernelEx(&cfg, KERNEL, mx, mw, p);
}

// ring slots compiled: 2, 3, 4, 6, 8 on one SM (k-chunk pairs or single
// chunks), 3 or 6 on a pair
template <int EPI>
static cudaError_t launch_1sm(int slots, cudaLaunchConfig_t& cfg, const CUtensorMap& mx, const CUtensorMap& mw,
                              const Params& p) {
    return slots == 8   ? launch_tile<gemm_kernel<EPI, 8>>(cfg, mx, mw, p)
           : slots == 6 ? launch_tile<gemm_kernel<EPI, 6>>(cfg, mx, mw, p)
           : slots == 4 ? launch_tile<gemm_kernel<EPI, 4>>(cfg, mx, mw, p)
           : slots == 3 ? launch_tile<gemm_kernel<EPI, 3>>(cfg, mx, mw, p)
                        : launch_tile<gemm_kernel<EPI, 2>>(cfg, mx, mw, p);
}
template <int EPI>
static cudaError_t launch_pair(int slots, cudaLaunchConfig_t& cfg, const CUtensorMap& mx, const CUtensorMap& mw,
                               const Params& p) {
    return slots == 6 ? launch_tile<gemm_pair_kernel<EPI, 6>>(cfg, mx, mw, p)
                      : launch_tile<gemm_pair_kernel<EPI, 3>>(cfg, mx, mw, p);
}

// [rows, K] bf16 seen as (64 k, row, k chunk): a box of box_rows rows and
// cps chunks lands as cps consecutive 128B-swizzled [box_rows x 64] tiles.
static bool make_map_kc(CUtensorMap* map, const void* base, int64_t rows, int64_t K, uint32_t box_rows, int cps) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)kKc, (cuuint64_t)rows, (cuuint64_t)(K / kKc)};
    const cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)kKc * 2};
    const cuuint32_t box[3] = {(cuuint32_t)kKc, box_rows, (cuuint32_t)cps};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// The stacked gate/up weights [2 I, K] as (64 k, row, half, k chunk): a box
// of bn rows, both halves and cps chunks lands per chunk as the bn gate rows
// followed by the bn up rows, the B operand of one N = 2 bn MMA.
static bool make_map_glu(CUtensorMap* map, const void* base, int64_t I, int64_t K, uint32_t bn, int cps) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[4] = {(cuuint64_t)kKc, (cuuint64_t)I, 2, (cuuint64_t)(K / kKc)};
    const cuuint64_t strides[3] = {(cuuint64_t)K * 2, (cuuint64_t)I * K * 2, (cuuint64_t)kKc * 2};
    const cuuint32_t box[4] = {(cuuint32_t)kKc, bn, 2, (cuuint32_t)cps};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static fg_status run(const void* x, int32_t M, int32_t K, const void* w, int32_t N, const void* bias,
                     const void* resid, int64_t ld_resid, void* out, int64_t ld_out, int32_t epi, int32_t bm,
                     int32_t bn, int32_t splits, int32_t stages, void* workspace, size_t workspace_bytes,
                     cudaStream_t stream) {
    const int sms = lmh::sm_count();
    resolve(M, N, K, epi, bm, bn, splits, stages);
    if (bm != kBM && bm != 2 * kBM) return FG_EINVAL;
    const bool pair = bm == 2 * kBM;
    if (!tile_ok(pair, bn, epi)) return FG_EINVAL;
    if (epi == FG_EPI_SWIGLU && N % bn) return FG_EINVAL;
    const int nb = epi == FG_EPI_SWIGLU ? 2 * bn : bn;
    // ring depths compiled: 4, 6 or 8 stages on one SM, 6 on a pair
    const bool st_ok = pair ? stages == kStagesPair : (stages == 4 || stages == 6 || stages == 8);
    if (!st_ok || stages > fit_stages(pair, nb)) return FG_EINVAL;
    Params p;
    p.M = M;
    p.N = N;
    p.K = K;
    p.bn = bn;
    p.nb = nb;
    p.n_mt = (M + bm - 1) / bm;
    p.n_nt = (N + bn - 1) / bn;
    p.nk = K / kKc;
    if (splits > p.nk) return FG_EINVAL;
    p.splits = splits;
    p.units = p.n_mt * p.n_nt * splits;
    // `stages` k chunks in flight, as ring slots of two chunks each when K
    // has an even number of chunks (one TMA instruction per operand and
    // stage moves twice the bytes: the per-SM ingest grows with the bytes per
    // instruction); as many two-chunk slots as fit, at least two
    p.cps = 1;
    int slots = stages;
    if (p.nk % 2 == 0 && splits <= p.nk / 2) {
        const int fit2 = (kSmemMax - 1024 - kOffStage) / (2 * stage_bytes(pair, nb));
        const int want = pair ? 3 : min(stages / 2, 4);
        if (fit2 >= 2) {
            p.cps = 2;
            slots = pair ? (fit2 >= 3 ? 3 : 0) : min(want, fit2);
            if (slots == 0) {
                p.cps = 1;
                slots = stages;
            }
        }
    }
    p.stage_bytes = p.cps * stage_bytes(pair, nb);
    p.bias = (const __nv_bfloat16*)bias;
    p.resid = (const __nv_bfloat16*)resid;
    p.ld_resid = ld_resid;
    p.out = (__nv_bfloat16*)out;
    p.ld_out = ld_out;
    p.ws = nullptr;
    if (splits > 1) {
        const size_t need = ws_bytes(M, N, epi, splits);
        if (!workspace || workspace_bytes < need || ((uintptr_t)workspace % 16)) return FG_ECAPACITY;
        p.ws = (float*)workspace;
    }
    // weight box rows: a whole tile on one SM; half of it per CTA of a pair
    // (SwiGLU: the gate rows on the even CTA, the up rows on the odd one)
    const int wbox = pair ? nb / 2 : bn;
    CUtensorMap mx, mw;
    const bool glu4 = epi == FG_EPI_SWIGLU && !pair;
    if (!make_map_kc(&mx, x, M, K, kBM, p.cps) ||
        !(glu4 ? make_map_glu(&mw, w, N, K, (uint32_t)bn, p.cps)
               : make_map_kc(&mw, w, epi == FG_EPI_SWIGLU ? 2 * (int64_t)N : N, K, (uint32_t)wbox, p.cps)))
        return FG_EINVAL;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = 1024 + kOffStage + slots * p.stage_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cudaError_t e;
    if (pair) {
        const int pairs = p.units < sms / 2 ? p.units : sms / 2;
        cfg.gridDim = dim3(2 * pairs);
        cfg.numAttrs = 2;
        e = epi == FG_EPI_STORE   ? launch_pair<FG_EPI_STORE>(slots, cfg, mx, mw, p)
            : epi == FG_EPI_RESID ? launch_pair<FG_EPI_RESID>(slots, cfg, mx, mw, p)
                                  : launch_pair<FG_EPI_SWIGLU>(slots, cfg, mx, mw, p);
    } else {
        cfg.gridDim = dim3(p.units < sms ? p.units : sms);
        cfg.numAttrs = 1;
        e = epi == FG_EPI_STORE   ? launch_1sm<FG_EPI_STORE>(slots, cfg, mx, mw, p)
            : epi == FG_EPI_RESID ? launch_1sm<FG_EPI_RESID>(slots, cfg, mx, mw, p)
                                  : launch_1sm<FG_EPI_SWIGLU>(slots, cfg, mx, mw, p);
    }
    if (e == cudaSuccess && splits > 1) {
        const int64_t items = (int64_t)M * (N / 8);
        const int64_t want = (items + 255) / 256;
        const int blocks = (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
        e = epi == FG_EPI_STORE   ? launch_pdl(linear_reduce_kernel<FG_EPI_STORE>, dim3(blocks), dim3(256), 0, stream, p)
            : epi == FG_EPI_RESID ? launch_pdl(linear_reduce_kernel<FG_EPI_RESID>, dim3(blocks), dim3(256), 0, stream, p)
                                  : launch_pdl(linear_reduce_kernel<FG_EPI_SWIGLU>, dim3(blocks), dim3(256), 0, stream, p);
    }
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return FG_ECUDA;
    }
    return launch_status();
}

static fg_status check(const void* x, int32_t dtype, int32_t M, int32_t K, const void* w, int32_t N, void* out,
                       int64_t ld_out) {
    if (dtype != FG_DTYPE_BF16) return FG_EUNSUPPORTED;
    if (!x || !w || !out || M < 0 || N <= 0 || K <= 0) return FG_EINVAL;
    if (K % kKc) return FG_ECAPACITY;
    if (N % 8 || ld_out < N || ld_out % 8) return FG_EINVAL;
    if (((uintptr_t)x % 16) || ((uintptr_t)w % 16) || ((uintptr_t)out % 16)) return FG_EINVAL;
    return FG_OK;
}

}  // namespace gemm
}  // namespace fg

extern "C" size_t fg_linear_workspace_size(int32_t M, int32_t N, int32_t K, int32_t epilogue, int32_t bm, int32_t bn,
                                           int32_t splits) {
    if (M <= 0 || N <= 0 || K <= 0 || K % gemm::kKc) return 0;
    int32_t stages = 2;
    gemm::resolve(M, N, K, epilogue, bm, bn, splits, stages);
    if (bm != gemm::kBM && bm != 2 * gemm::kBM) return 0;
    return gemm::ws_bytes(M, N, epilogue, splits);
}

extern "C" fg_status fg_linear(const void* x, int32_t dtype, int32_t M, int32_t K, const void* w, int32_t N,
                               const void* bias, const void* resid, int64_t ld_resid, void* out, int64_t ld_out,
                               int32_t epilogue, int32_t bm, int32_t bn, int32_t splits, int32_t stages,
                               void* workspace, size_t workspace_bytes, void* stream) {
    if (M == 0) return FG_OK;
    const fg_status st = gemm::check(x, dtype, M, K, w, N, out, ld_out);
    if (st != FG_OK) return st;
    if (epilogue != FG_EPI_STORE && epilogue != FG_EPI_RESID && epilogue != FG_EPI_SWIGLU) return FG_EINVAL;
    if (bias && ((uintptr_t)bias % 16)) return FG_EINVAL;
    if (epilogue == FG_EPI_RESID && (!resid || ((uintptr_t)resid % 16) || ld_resid < N || ld_resid % 8))
        return FG_EINVAL;
    if (epilogue == FG_EPI_SWIGLU && bias) return FG_EINVAL;
    return gemm::run(x, M, K, w, N, bias, resid, ld_resid, out, ld_out, epilogue, bm, bn, splits, stages, workspace,
                     workspace_bytes, (cudaStream_t)stream);
}

extern "C" fg_status fg_gate_up_silu(const void* x, int32_t dtype, int32_t T, int32_t H, const void* w_gate_up,
                                     int32_t I, void* out, void* stream) {
    if (T == 0) return FG_OK;
    if (dtype == FG_DTYPE_BF16 && I % 16) return FG_ECAPACITY;
    const fg_status st = gemm::check(x, dtype, T, H, w_gate_up, I, out, I);
    if (st != FG_OK) return st;
    // one k range per tile: the fused MLP needs no workspace
    int32_t bm = 0, bn = 0, splits = 1, stages = 0;
    gemm::resolve(T, I, H, FG_EPI_SWIGLU, bm, bn, splits, stages);
    return gemm::run(x, T, H, w_gate_up, I, nullptr, nullptr, 0, out, I, FG_EPI_SWIGLU, bm, bn, 1, stages, nullptr, 0,
                     (cudaStream_t)stream);
}

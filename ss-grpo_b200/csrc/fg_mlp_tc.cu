// fg_mlp_tc.cu -- the verify forward's gate/up projection with SwiGLU in the
// epilogue, on the tensor cores.
//
// act[t, j] = bf16(bf16(silu(bf16(g))) * bf16(u)),  g = X[t] . W[j],  u = X[t] . W[I + j]
// for X [T, H] (the post-attention RMSNorm output), W = [gate_proj; up_proj]
// [2I, H] bf16: the Qwen2 / Llama MLP's act_fn(gate_proj(x)) * up_proj(x)
// with every torch op's bf16 rounding, as fg_silu_mul applies it to a
// materialized gate/up tensor -- which this kernel never writes.
//
// Tiles: 128 tokens x BN outputs (BN a multiple of 16, at most 128, chosen
// per call so the tiles fill the last wave of the grid: 112 for I = 8960).
// The B operand of a tile is the BN gate rows stacked on the matching BN up
// rows (two TMA boxes), so one N = 2 BN tcgen05.mma per 16-wide k step puts
// gate and up of output j in the same TMEM lane, BN columns apart.  Persistent grid (one CTA per SM, tiles
// round-robin, ordered weight-tile-major so the token tiles of one weight
// tile run together and the weights stream from HBM about once):
//   warp 0     TMA: per 64-wide k chunk the X box (128 x 64) and the two
//              weight boxes into a 4-stage ring (up to 48 KB per stage,
//              128-byte swizzle);
//   warp 1     allocates 512 TMEM columns = two accumulators at columns 0
//              and 256;
//              one thread issues the MMAs, commits stages and tiles;
//   warps 4-11 epilogue: warp w reads TMEM lanes 32 (w % 4).. (one token
//              row per thread) and output half (w - 4) / 4 of the tile,
//              applies SiLU-gating and stores bf16 rows; the accumulator is
//              released to the MMA warp as soon as it is read, so the
//              epilogue of tile i overlaps the MMAs of tile i + 1.
// Every mbarrier wait is bounded (about one second).
#include "fg_common.cuh"

namespace fg {
namespace mlp {

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

constexpr int kBM = 128;                    // tokens per tile
constexpr int kBN = 128;                    // largest outputs per tile (gate + up = MMA N 256)
constexpr int kKc = 64;                     // k elements per stage (128-byte rows)
constexpr int kStages = 4;
constexpr int kThreads = 384;
constexpr int kABytes = kBM * 128;          // 16 KB
constexpr int kBBytes = 2 * kBN * 128;      // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kOffStage = 1024;             // barriers in the first 1 KB
constexpr int kSmemBytes = 1024 + kOffStage + kStages * kStageBytes;
constexpr uint32_t kTmemCols = 512;

struct Params {
    int32_t T, H, I;
    int32_t bn;  // outputs per tile
    int32_t n_mt, n_tiles, nk;
    __nv_bfloat16* out;  // [T, I]
};

struct Bars {
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
};

__global__ void __launch_bounds__(kThreads, 1) gate_up_silu_kernel(const __grid_constant__ CUtensorMap tmX,
                                                                   const __grid_constant__ CUtensorMap tmW, Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem);
    volatile int* abort_flag = &bars->abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // tiles of this CTA: blockIdx.x, blockIdx.x + gridDim.x, ...
    const int my_tiles = p.n_tiles > (int)blockIdx.x ? (p.n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
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
            const uint64_t pol_w = lmh::policy_evict_first(), pol_x = lmh::policy_evict_last();
            int it = 0, issued = 0;
            bool ok = true;
            for (int i = 0; i < my_tiles && ok; ++i) {
                const int tile = (int)blockIdx.x + i * (int)gridDim.x;
                const int nt = tile / p.n_mt, mt = tile - nt * p.n_mt;
                for (int kc = 0; kc < p.nk; ++kc, ++it) {
                    const int s = it % kStages;
                    if (it >= kStages && !(ok = bar_wait(&bars->empty[s], ((it / kStages) - 1) & 1, abort_flag)))
                        break;
                    uint8_t* st = smem + kOffStage + s * kStageBytes;
                    bar_expect(&bars->full[s], (uint32_t)(kABytes + 2 * p.bn * 128));
                    lmh::tma_2d(st, &tmX, kc * kKc, mt * kBM, &bars->full[s], pol_x);
                    lmh::tma_2d(st + kABytes, &tmW, kc * kKc, nt * p.bn, &bars->full[s], pol_w);
                    lmh::tma_2d(st + kABytes + p.bn * 128, &tmW, kc * kKc, p.I + nt * p.bn, &bars->full[s], pol_w);
                    issued = it + 1;
                }
            }
            for (int j = max(0, issued - kStages); j < issued; ++j)
                bar_drain(&bars->full[j % kStages], (j / kStages) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_bf16(2 * p.bn, false);
            int it = 0;
            bool ok = true;
            for (int i = 0; i < my_tiles && ok; ++i) {
                const int a = i & 1;
                if (i >= 2 && !(ok = bar_wait(&bars->acc_empty[a], ((i >> 1) - 1) & 1, abort_flag))) break;
                fence_after();
                for (int kc = 0; kc < p.nk; ++kc, ++it) {
                    const int s = it % kStages;
                    if (!(ok = bar_wait(&bars->full[s], (it / kStages) & 1, abort_flag))) break;
                    fence_after();
                    const uint32_t a_addr = sa(smem + kOffStage + s * kStageBytes);
                    const uint32_t b_addr = a_addr + (uint32_t)kABytes;
#pragma unroll
                    for (int kk = 0; kk < kKc / 16; ++kk) {
                        const uint64_t da = sdesc(a_addr + kk * 32, 16, 1024);
                        const uint64_t db = sdesc(b_addr + kk * 32, 16, 1024);
                        umma(tmem + (uint32_t)(a * 256), da, db, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
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
        const int q4 = warp & 3, h = (warp - 4) >> 2;
        const uint32_t lane_addr = tmem + ((uint32_t)(q4 * 32) << 16);
        for (int i = 0; i < my_tiles; ++i) {
            const int a = i & 1;
            if (!__all_sync(0xffffffffu, bar_wait(&bars->acc_full[a], (i >> 1) & 1, abort_flag))) break;
            fence_after();
            const int tile = (int)blockIdx.x + i * (int)gridDim.x;
            const int nt = tile / p.n_mt, mt = tile - nt * p.n_mt;
            const int row = mt * kBM + q4 * 32 + lane;
            const int half = p.bn / 2;  // outputs of this warp: [h half, (h + 1) half), a multiple of 8
            __nv_bfloat16* dst = p.out + (int64_t)row * p.I + nt * p.bn + h * half;
            // 32-column reads; past `half` they stay inside this accumulator's
            // 256 columns (bn + half + 32 * ceil(half / 32) <= 256) and are dropped
#pragma unroll 1
            for (int c = 0; c < half; c += 32) {
                float g[32], u[32];
                tld32(lane_addr + (uint32_t)(a * 256 + h * half + c), g);
                tld32(lane_addr + (uint32_t)(a * 256 + p.bn + h * half + c), u);
                const int n8 = min(32, half - c) / 8;
                if (row < p.T) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        if (q >= n8) break;
                        uint4 v;
                        uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            float o[2];
#pragma unroll
                            for (int z = 0; z < 2; ++z) {
                                const int j = 8 * q + 2 * e + z;
                                const float gb = rnd<__nv_bfloat16>(g[j]), ub = rnd<__nv_bfloat16>(u[j]);
                                o[z] = rnd<__nv_bfloat16>(silu(gb)) * ub;
                            }
                            w[e] = tc::pack2(o[0], o[1]);
                        }
                        *reinterpret_cast<uint4*>(dst + c + 8 * q) = v;
                    }
                }
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

}  // namespace mlp
}  // namespace fg

extern "C" fg_status fg_gate_up_silu(const void* x, int32_t dtype, int32_t T, int32_t H, const void* w_gate_up,
                                     int32_t I, void* out, void* stream) {
    if (T == 0) return FG_OK;
    if (dtype != FG_DTYPE_BF16) return FG_EUNSUPPORTED;
    if (!x || !w_gate_up || !out || T < 0 || H <= 0 || I <= 0) return FG_EINVAL;
    if (H % mlp::kKc || I % 16) return FG_ECAPACITY;
    if (((uintptr_t)x % 16) || ((uintptr_t)w_gate_up % 16) || ((uintptr_t)out % 16)) return FG_EINVAL;
    mlp::Params p;
    p.T = T;
    p.H = H;
    p.I = I;
    p.n_mt = (T + mlp::kBM - 1) / mlp::kBM;
    // outputs per tile: the candidate dividing I whose tiles fill the grid's
    // waves best (cost = waves x (bn + a fixed per-tile share))
    const int sms = lmh::sm_count();
    p.bn = 0;
    int64_t best = 0;
    for (int bn = mlp::kBN; bn >= 16; bn -= 16) {
        if (I % bn) continue;
        const int64_t tiles = (int64_t)p.n_mt * (I / bn);
        const int64_t cost = (tiles + sms - 1) / sms * (bn + 16);
        if (p.bn == 0 || cost < best) {
            p.bn = bn;
            best = cost;
        }
    }
    p.n_tiles = p.n_mt * (I / p.bn);
    p.nk = H / mlp::kKc;
    p.out = (__nv_bfloat16*)out;
    CUtensorMap mx, mw;
    if (!lmh::make_map_2d(&mx, x, H, T, H, mlp::kBM) ||
        !lmh::make_map_2d(&mw, w_gate_up, H, 2 * (int64_t)I, H, (uint32_t)p.bn))
        return FG_EINVAL;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(mlp::gate_up_silu_kernel,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, mlp::kSmemBytes);
        if (e != cudaSuccess) {
            set_cuda_error(e);
            return FG_ECUDA;
        }
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const int grid = p.n_tiles < sms ? p.n_tiles : sms;
    mlp::gate_up_silu_kernel<<<grid, mlp::kThreads, mlp::kSmemBytes, (cudaStream_t)stream>>>(mx, mw, p);
    return launch_status();
}

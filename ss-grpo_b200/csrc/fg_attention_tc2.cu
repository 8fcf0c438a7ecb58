// fg_attention_tc2.cu -- K3 for wide query groups: 256 query rows per CTA.
//
// The bf16 tree attention of fg_attention_tc.cu for KV heads with 129-256
// query rows (N x G: the 7B / 8B-shaped trees, the N = 64 points of the
// attention sweep), near the ridge where the tensor pipe starts to bound.
// Each K/V tile now serves two 128-row query halves A and B, so the slots
// stream through shared memory once per 256 rows, and P stays in TMEM:
//   warp 0 / warp 2   TMA producers of the K and V tiles (2-stage ring of
//                     128-slot tiles; a stage's K half is released after both
//                     halves' QK, its V half after both halves' PV);
//   warp 1            one thread issues per KV tile i: S_A = Q_A K^T and
//                     S_B = Q_B K^T (M = 128, N = 128 slots, K = 128 dims)
//                     into TMEM, then O_h += P_h V with P_h read from TMEM
//                     (the TS form of tcgen05.mma: P_h overwrites the first
//                     64 columns of S_h as packed bf16 pairs).  Issue order
//                     QK_A(0) QK_B(0) | PV_A(i) QK_A(i+1) PV_B(i) QK_B(i+1)
//                     ...: the tensor pipe runs a thread's MMAs in issue
//                     order, so QK_h(i+1) overwrites S_h only after PV_h(i)
//                     has read P_h(i), and the softmax of one half overlaps
//                     the other half's MMAs;
//   warps 4-7 / 8-11  the online softmax of half A / half B over every tile:
//                     tcgen05.ld of S_h, tree mask, log2-domain exponentials
//                     with lazy rescaling of O_h in TMEM, P_h as bf16 into
//                     TMEM (tcgen05.st); each half finishes its own rows (no
//                     merge between halves).
// With several splits each half writes (O, m, l) partials as its own
// 128-row sub-item (2 x item + half) and the last CTA of the item merges both
// sub-items.  Every mbarrier wait is bounded, as in fg_attention_tc.cu.
#include "fg_common.cuh"

namespace fg {
namespace tc {

constexpr int kWideRows = 256;                                  // query rows per CTA (two halves)
constexpr int kWOffStage = 2 * kQBytes;                         // Q_A, Q_B: 64 KB
constexpr int kWOffBar = kWOffStage + kStages * kStageBytes;    // 192 KB
constexpr int kWSmemBytes = kWOffBar + 256 + 1024;
static_assert(2 * kMaxSplits * kRows * 4 <= kWOffBar, "split (m, l) tables fit below the barriers");

struct WideBars {
    uint64_t k_full[kStages];
    uint64_t k_empty[kStages];
    uint64_t v_full[kStages];
    uint64_t v_empty[kStages];
    uint64_t s_full[2];   // per half: S_h of the next tile is in TMEM
    uint64_t p_full[2];   // per half: P_h written (4 warp arrivals)
    uint64_t o_done[2];   // per half: PV_h completed
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
    int last_flag;
};

// A = P from TMEM (32-bit columns, bf16 pairs along K), B from shared memory.
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

// 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tst16u(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// The last CTA of an item merges the splits of one 128-row sub-item (rows
// [rowbase, rowbase + rs) of the KV head): per row the weights
// exp2(m_s - m) / l over the splits, then the weighted sum of the fp32
// partials, written as bf16.
__device__ void merge_sub_item(const Params& p, int sub, int rowbase, int rs, int b, int kvh, uint8_t* smem) {
    const float* wo_all = p.ws_o + (int64_t)sub * p.splits * (kRows * kD);
    const float* wml_all = p.ws_ml + (int64_t)sub * p.splits * (2 * kRows);
    float* wt = reinterpret_cast<float*>(smem);  // [split][row]
    float* ls = wt + p.splits * kRows;           // [split][row]
    for (int e = threadIdx.x; e < p.splits * rs; e += blockDim.x) {
        const int s2 = e / rs, rw = e - s2 * rs;
        wt[s2 * kRows + rw] = __ldcg(wml_all + s2 * 2 * kRows + rw);
        ls[s2 * kRows + rw] = __ldcg(wml_all + s2 * 2 * kRows + kRows + rw);
    }
    __syncthreads();
    for (int rw = threadIdx.x; rw < rs; rw += blockDim.x) {
        float mt = -INFINITY;
        for (int s2 = 0; s2 < p.splits; ++s2) mt = fmaxf(mt, wt[s2 * kRows + rw]);
        float lt = 0.0f;
        for (int s2 = 0; s2 < p.splits; ++s2) {
            const float ms = wt[s2 * kRows + rw];
            const float w = (ms == -INFINITY) ? 0.0f : ex2(ms - mt);
            lt += w * ls[s2 * kRows + rw];
            wt[s2 * kRows + rw] = w;
        }
        const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
        for (int s2 = 0; s2 < p.splits; ++s2) wt[s2 * kRows + rw] *= inv;
    }
    __syncthreads();
    const int total = rs * (kD / 4);
    for (int e0 = threadIdx.x; e0 < total; e0 += 4 * blockDim.x) {
        float4 acc[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 2
        for (int s2 = 0; s2 < p.splits; ++s2) {
            float4 v[4];
            float w[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = min(e0 + u * (int)blockDim.x, total - 1);
                const int rw = e / (kD / 4), d = (e % (kD / 4)) * 4;
                v[u] = __ldcg(reinterpret_cast<const float4*>(wo_all + (int64_t)s2 * kRows * kD + rw * kD + d));
                w[u] = wt[s2 * kRows + rw];
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                acc[u].x = fmaf(w[u], v[u].x, acc[u].x);
                acc[u].y = fmaf(w[u], v[u].y, acc[u].y);
                acc[u].z = fmaf(w[u], v[u].z, acc[u].z);
                acc[u].w = fmaf(w[u], v[u].w, acc[u].w);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int e = e0 + u * (int)blockDim.x;
            if (e < total) {
                const int rw = e / (kD / 4), d = (e % (kD / 4)) * 4;
                const int rr = rowbase + rw;
                __nv_bfloat16* orow = p.out + (((int64_t)b * p.N + rr / p.G) * p.Hq + kvh * p.G + rr % p.G) * kD;
                uint2 pk;
                pk.x = pack2(acc[u].x, acc[u].y);
                pk.y = pack2(acc[u].z, acc[u].w);
                *reinterpret_cast<uint2*>(orow + d) = pk;
            }
        }
    }
    __syncthreads();  // the (m, l) tables are reused by the next sub-item
}

__global__ void __launch_bounds__(kThreads, 1) attn_tc_wide_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                   const __grid_constant__ CUtensorMap tmV, Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    WideBars* bars = reinterpret_cast<WideBars*>(smem + kWOffBar);
    volatile int* abort_flag = &bars->abort_flag;

    const int split = blockIdx.x;
    const int kvh = blockIdx.y / p.groups, grp = blockIdx.y % p.groups;  // p.groups: 256-row groups
    const int b = blockIdx.z;
    const int bkv = max(cache_row(p.kv_rows, p.kv_batch, b), 0);
    const int row0 = grp * kWideRows;
    const int R = min(kWideRows, p.rows_total - row0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kv_len = p.kv_len[b];
    const int T = kv_len + p.N;
    const int nblk = (T + kBlk - 1) / kBlk;
    const int per = (nblk + p.splits - 1) / p.splits;
    const int c0 = min(nblk, split * per);
    const int nmine = min(nblk, c0 + per) - c0;
    const int item = (b * p.Hkv + kvh) * p.groups + grp;

    auto load_k = [&](int i) {
        const int s = i % kStages;
        uint8_t* st = smem + kWOffStage + s * kStageBytes;
        const int slot = (c0 + i) * kBlk;
        bar_expect(&bars->k_full[s], 2 * kBox);
        tma_4d(st, &tmK, 0, slot, kvh, bkv, &bars->k_full[s]);
        tma_4d(st + kBox, &tmK, 64, slot, kvh, bkv, &bars->k_full[s]);
    };
    auto load_v = [&](int i) {
        const int s = i % kStages;
        uint8_t* st = smem + kWOffStage + s * kStageBytes + 2 * kBox;
        const int slot = (c0 + i) * kBlk;
        bar_expect(&bars->v_full[s], 2 * kBox);
        tma_4d(st, &tmV, 0, slot, kvh, bkv, &bars->v_full[s]);
        tma_4d(st + kBox, &tmV, 64, slot, kvh, bkv, &bars->v_full[s]);
    };
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            bar_init(&bars->k_full[s], 1);
            bar_init(&bars->k_empty[s], 1);
            bar_init(&bars->v_full[s], 1);
            bar_init(&bars->v_empty[s], 1);
        }
        for (int h = 0; h < 2; ++h) {
            bar_init(&bars->s_full[h], 1);
            bar_init(&bars->p_full[h], 4);
            bar_init(&bars->o_done[h], 1);
        }
        bar_init(&bars->drain, 1);
        bars->abort_flag = 0;
        bars->last_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // prefix tiles (written by earlier rounds) load before the grid
        // dependency wait; tiles reaching the tree slots after it
        for (int i = 0; i < min(kStages, nmine); ++i)
            if ((c0 + i + 1) * kBlk <= kv_len) {
                load_k(i);
                load_v(i);
            }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(&bars->tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0)
        for (int i = 0; i < min(kStages, nmine); ++i)
            if ((c0 + i + 1) * kBlk > kv_len) {
                load_k(i);
                load_v(i);
            }
    const int h = warp >= 4 ? (warp - 4) >> 2 : -1;  // softmax half (A = 0, B = 1)
    const int r = (warp & 3) * 32 + lane;             // row within the half = TMEM lane
    // Q half h (rows beyond R zero) -> swizzled smem: two 64-dim halves of
    // 128 rows x 128 bytes each, as the QK descriptors read them
    if (h >= 0) {
        uint8_t* qs = smem + h * kQBytes;
        const int hr = h * kRows + r;
        const bool valid = hr < R;
        const int rr = row0 + (valid ? hr : 0);
        const __nv_bfloat16* qrow = p.q + (((int64_t)b * p.N + rr / p.G) * p.Hq + kvh * p.G + rr % p.G) * kD;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            const uint4 v = valid ? *reinterpret_cast<const uint4*>(qrow + c * 8) : make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(qs + (c >> 3) * (kRows * 128) + sw128(r, c & 7)) = v;
        }
        fence_async_smem();
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0 || warp == 2) {
        // ------------------------------------- TMA producers: K (warp 0), V (warp 2)
        if (lane == 0) {
            const bool is_k = warp == 0;
            uint64_t* empty = is_k ? bars->k_empty : bars->v_empty;
            uint64_t* full = is_k ? bars->k_full : bars->v_full;
            int issued = min(kStages, nmine);
            for (int i = kStages; i < nmine; ++i) {
                const int s = i % kStages;
                if (!bar_wait(&empty[s], ((i / kStages) - 1) & 1, abort_flag)) break;
                if (is_k) load_k(i); else load_v(i);
                issued = i + 1;
            }
            for (int j = max(0, issued - kStages); j < issued; ++j) bar_drain(&full[j % kStages], (j / kStages) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t id_qk = idesc_bf16(kBlk, false);
            constexpr uint32_t id_pv = idesc_bf16(kD, true);
            bool ok = true;
            auto qk = [&](int hh, int i) {
                if (!ok || !(ok = bar_wait(&bars->k_full[i % kStages], (i / kStages) & 1, abort_flag))) return;
                fence_after();
                const uint32_t q_addr = sa(smem + hh * kQBytes);
                const uint32_t k_addr = sa(smem + kWOffStage + (i % kStages) * kStageBytes);
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk) {
                    const uint64_t da = sdesc(q_addr + (kk >> 2) * (kRows * 128) + (kk & 3) * 32, 16, 1024);
                    const uint64_t db = sdesc(k_addr + (kk >> 2) * kBox + (kk & 3) * 32, 16, 1024);
                    umma(tmem + (uint32_t)(hh * kBlk), da, db, id_qk, kk > 0 ? 1u : 0u);
                }
                umma_commit(&bars->s_full[hh]);
                if (hh == 1) umma_commit(&bars->k_empty[i % kStages]);  // both halves' QK(i) done
            };
            auto pv = [&](int hh, int i) {
                if (!ok || !(ok = bar_wait(&bars->v_full[i % kStages], (i / kStages) & 1, abort_flag))) return;
                if (!(ok = bar_wait(&bars->p_full[hh], i & 1, abort_flag))) return;
                fence_after();
                const uint32_t v_addr = sa(smem + kWOffStage + (i % kStages) * kStageBytes + 2 * kBox);
                const uint32_t o_col = kColO0 + (uint32_t)hh * kD;
#pragma unroll
                for (int kk = 0; kk < kBlk / 16; ++kk) {
                    const uint64_t db = sdesc(v_addr + kk * 2048, kBox, 1024);
                    // P_h: 8 columns of bf16 pairs per 16-slot k step
                    umma_ts(tmem + o_col, tmem + (uint32_t)(hh * kBlk + kk * 8), db, id_pv,
                            (i > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(&bars->o_done[hh]);
                if (hh == 1) umma_commit(&bars->v_empty[i % kStages]);  // both halves' PV(i) done
            };
            if (nmine > 0) {
                qk(0, 0);
                qk(1, 0);
            }
            for (int i = 0; i < nmine && ok; ++i) {
                pv(0, i);
                if (i + 1 < nmine) qk(0, i + 1);
                pv(1, i);
                if (i + 1 < nmine) qk(1, i + 1);
            }
            if (!ok) {
                *abort_flag = 1;
                atomicCAS(&g_fg_error_word, 0, FG_ETIMEOUT);
            }
            // everything issued has completed before TMEM is read or freed
            umma_commit(&bars->drain);
            bar_drain(&bars->drain, 0);
        }
    } else if (h >= 0) {
        // ------------------------------------------- softmax of half h
        const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t s_col = (uint32_t)(h * kBlk);
        const uint32_t o_col = kColO0 + (uint32_t)h * kD;
        const int hr = h * kRows + r;
        const bool valid = hr < R;
        const int rr = row0 + (valid ? hr : 0);
        const int node = rr / p.G;
        uint32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
        if (valid) {
            a0 = p.anc[node * 4 + 0];
            a1 = p.anc[node * 4 + 1];
            a2 = p.anc[node * 4 + 2];
            a3 = p.anc[node * 4 + 3];
        }
        float m_used = -INFINITY, l = 0.0f;
        bool ok = true;
        constexpr unsigned kFull = 0xffffffffu;
        for (int i = 0; i < nmine; ++i) {
            if (!__all_sync(kFull, bar_wait(&bars->s_full[h], i & 1, abort_flag))) {
                ok = false;
                break;
            }
            fence_after();
            float sv[kBlk];
            tld128(tmem + lane_addr + s_col, sv);
            const int base = (c0 + i) * kBlk;
            if (base + kBlk > kv_len) {
                uint32_t vis[kBlk / 32];
#pragma unroll
                for (int w = 0; w < kBlk / 32; ++w) vis[w] = visible_bits(base + 32 * w, kv_len, T, a0, a1, a2, a3);
#pragma unroll
                for (int c = 0; c < kBlk; ++c) sv[c] = ((vis[c >> 5] >> (c & 31)) & 1u) ? sv[c] : -INFINITY;
            }
            float mq0 = sv[0], mq1 = sv[1], mq2 = sv[2], mq3 = sv[3];
#pragma unroll
            for (int c = 4; c < kBlk; c += 4) {
                mq0 = fmaxf(mq0, sv[c]);
                mq1 = fmaxf(mq1, sv[c + 1]);
                mq2 = fmaxf(mq2, sv[c + 2]);
                mq3 = fmaxf(mq3, sv[c + 3]);
            }
            const float mx = fmaxf(fmaxf(mq0, mq1), fmaxf(mq2, mq3)) * p.scale_log2;
            // QK_h(i) completed after PV_h(i - 1) (issue order), so O_h is stable
            const bool grow = mx > m_used + kRescaleLog2 || (m_used == -INFINITY && mx != -INFINITY);
            const float alpha = grow ? ((m_used == -INFINITY) ? 0.0f : ex2(m_used - mx)) : 1.0f;
            const bool rescale_o = i >= 1 && __any_sync(kFull, grow);
            if (grow) {
                l *= alpha;
                m_used = mx;
            }
            // P_h = exp2(s - m_used) as bf16 pairs over the first 64 columns of S_h
            const float mneg = m_used == -INFINITY ? 0.0f : -m_used;
            float rs0 = 0.0f, rs1 = 0.0f;
#pragma unroll
            for (int c0c = 0; c0c < kBlk; c0c += 32) {
                uint32_t pk[16];
#pragma unroll
                for (int c = 0; c < 32; c += 8) {
                    float e[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) e[q] = ex2(fmaf(sv[c0c + c + q], p.scale_log2, mneg));
                    const float part = ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
                    if ((c >> 3) & 1) rs1 += part; else rs0 += part;
#pragma unroll
                    for (int q = 0; q < 8; q += 2) pk[(c + q) >> 1] = pack2(e[q], e[q + 1]);
                }
                tst16u(tmem + lane_addr + s_col + (uint32_t)(c0c >> 1), pk);
            }
            l += rs0 + rs1;
            if (rescale_o) {
#pragma unroll 1
                for (int cch = 0; cch < kD; cch += 32) {
                    float ov[32];
                    tld32(tmem + lane_addr + o_col + cch, ov);
#pragma unroll
                    for (int c = 0; c < 32; ++c) ov[c] *= alpha;
                    tst32(tmem + lane_addr + o_col + cch, ov);
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&bars->p_full[h]);
        }
        // ---- epilogue: this half's last PV, then its rows
        if (ok && nmine > 0) ok = __all_sync(kFull, bar_wait(&bars->o_done[h], (nmine - 1) & 1, abort_flag));
        fence_after();
        const int aborted = *abort_flag;
        if (__all_sync(kFull, ok) && !__any_sync(kFull, aborted != 0)) {
            float* wo = nullptr;
            const int sub = 2 * item + h;
            if (p.splits > 1) {
                wo = p.ws_o + ((int64_t)sub * p.splits + split) * (kRows * kD) + (int64_t)r * kD;
                float* wml = p.ws_ml + ((int64_t)sub * p.splits + split) * (2 * kRows);
                wml[r] = (nmine > 0 && l > 0.0f) ? m_used : -INFINITY;
                wml[kRows + r] = nmine > 0 ? l : 0.0f;
            }
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            __nv_bfloat16* orow = p.out + (((int64_t)b * p.N + rr / p.G) * p.Hq + kvh * p.G + rr % p.G) * kD;
#pragma unroll 1
            for (int cch = 0; cch < kD; cch += 32) {
                float oa[32];
                if (nmine > 0) {
                    tld32(tmem + lane_addr + o_col + cch, oa);
                } else {
#pragma unroll
                    for (int c = 0; c < 32; ++c) oa[c] = 0.0f;
                }
                if (p.splits == 1) {
                    if (valid) {
#pragma unroll
                        for (int c = 0; c < 32; c += 8) {
                            uint4 w;
                            w.x = pack2(oa[c] * inv, oa[c + 1] * inv);
                            w.y = pack2(oa[c + 2] * inv, oa[c + 3] * inv);
                            w.z = pack2(oa[c + 4] * inv, oa[c + 5] * inv);
                            w.w = pack2(oa[c + 6] * inv, oa[c + 7] * inv);
                            *reinterpret_cast<uint4*>(orow + cch + c) = w;
                        }
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < 32; c += 4)
                        *reinterpret_cast<float4*>(wo + cch + c) = make_float4(oa[c], oa[c + 1], oa[c + 2], oa[c + 3]);
                }
            }
        }
        fence_before();
    }
    // ---- all roles done with TMEM: free it; splits merge below
    __syncthreads();
    fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    if (p.splits == 1 || *abort_flag) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(&p.ws_cnt[item], 1);
        bars->last_flag = (prev == p.splits - 1) ? 1 : 0;
    }
    __syncthreads();
    if (!bars->last_flag) return;
    __threadfence();
    merge_sub_item(p, 2 * item, row0, min(kRows, R), b, kvh, smem);
    if (R > kRows) merge_sub_item(p, 2 * item + 1, row0 + kRows, R - kRows, b, kvh, smem);
    if (threadIdx.x == 0) p.ws_cnt[item] = 0;
}

}  // namespace tc
}  // namespace fg

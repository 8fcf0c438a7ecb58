// fg_attention.cu -- K3: flash-decoding GQA attention of the tree queries.
//
// Replaces the HF eager/SDPA attention with the dense additive 4D mask that
// forward_tree runs (flashgrpo_b200/models/qwen_flashgrpo_wrapper.py:220-239,
// mask from flashgrpo_b200/decoding/tree_attention.py:6-67).
//
// bf16 path (head_dim 128).  Grid (split, kv_head x row_group, row).  A CTA
// owns the query rows of one KV head -- row r = node * G + g, up to 128 rows --
// and streams its share of the row's KV slots [0, kv_len + n_nodes):
//   * one producer warp issues TMA tile loads (4-D tensor maps over
//     [B, Hkv, capacity, D], 64 slots x 64 dims per box, 128-byte swizzle)
//     into a 3-stage ring guarded by mbarriers (bounded waits);
//   * consumer warps (16 rows each) run S = Q K^T and O += P V on the tensor
//     cores (mma.m16n8k16 bf16, fp32 accumulators, Q and P held in
//     registers), an online softmax in the log2 domain, and the tree mask:
//     prefix slots are visible to every node, tree slot j to node i iff bit j
//     of anc_bits[i];
//   * with several splits, each CTA writes (O, m, l) partials and the last
//     CTA of a (row, head, group) merges them (a counter in the workspace
//     that the merging CTA resets to zero).
// f32 path: one warp per query head, exact fp32 dot products (parity checks
// of the fp32 configuration).
#include <cstdio>

#include "fg_common.cuh"

// g_fg_error_word is defined in fg_abi.cu (same translation unit).

namespace fg {

constexpr int kD = 128;
constexpr int kBlockN = 64;
constexpr int kStages = 3;
constexpr int kMaxRows = 128;
constexpr int kBoxBytes = 64 * 64 * 2;       // 64 slots x 64 dims bf16
constexpr int kStageBytes = 4 * kBoxBytes;   // K lo/hi, V lo/hi
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 64;
constexpr int64_t kWaitNs = 1000000000LL;    // 1 s bound on any barrier wait

struct AttnParams {
    const __nv_bfloat16* q;
    __nv_bfloat16* out;
    const int32_t* kv_len;
    const uint32_t* anc;
    int32_t N, Hq, Hkv, G, groups, splits, rows_total;
    float scale_log2;
    float* ws_o;      // [items][splits][128][128]
    float* ws_ml;     // [items][splits][2][128]
    int32_t* ws_cnt;  // [items]
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t addr, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    return done != 0;
}

// Returns false when the phase did not complete within kWaitNs.  The clock
// is only read once the barrier has stayed closed for a while, so the
// common path is a plain try_wait loop.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t addr = smem_u32(bar);
    for (int it = 0; it < 4096; ++it)
        if (mbar_try(addr, parity)) return true;
    const uint64_t start = now_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try(addr, parity)) return true;
        if ((it & 1023u) == 0u && (int64_t)(now_ns() - start) > kWaitNs) return false;
    }
}

// bit j (0..127) of a 4-word ancestor mask held in registers
__device__ __forceinline__ bool anc_bit(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, int j) {
    const uint32_t w = j < 64 ? (j < 32 ? a0 : a1) : (j < 96 ? a2 : a3);
    return (w >> (j & 31)) & 1u;
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// Byte offset of (slot, 16-byte column) inside one 64x64 bf16 box written by
// TMA with 128-byte swizzle: the column index is XORed with slot % 8.
__device__ __forceinline__ uint32_t swz(int slot, int col16) {
    return (uint32_t)(slot * 128 + ((col16 ^ (slot & 7)) << 4));
}

__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__global__ void __launch_bounds__(288, 1) tree_attn_bf16_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                const __grid_constant__ CUtensorMap tmV,
                                                                AttnParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    int32_t* flag = reinterpret_cast<int32_t*>(empty + kStages);

    const int split = blockIdx.x;
    const int kvh = blockIdx.y / p.groups, grp = blockIdx.y % p.groups;
    const int b = blockIdx.z;
    const int row0 = grp * kMaxRows;
    const int R = min(kMaxRows, p.rows_total - row0);
    const int WM = (R + 15) >> 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kv_len = p.kv_len[b];
    const int T = kv_len + p.N;
    const int nchunks = (T + kBlockN - 1) / kBlockN;
    const int cps = (nchunks + p.splits - 1) / p.splits;
    const int c_begin = min(nchunks, split * cps);
    const int c_end = min(nchunks, c_begin + cps);
    const int nmine = c_end - c_begin;
    const int item = (b * p.Hkv + kvh) * p.groups + grp;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], WM);
        }
        *flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (warp > WM) return;

    if (warp == WM) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            for (int i = 0; i < nmine; ++i) {
                const int s = i % kStages;
                if (i >= kStages && !mbar_wait(&empty[s], ((i / kStages) - 1) & 1)) {
                    atomicCAS(&g_fg_error_word, 0, FG_ETIMEOUT);
                    break;
                }
                uint8_t* st = smem + s * kStageBytes;
                const int slot = (c_begin + i) * kBlockN;
                mbar_expect_tx(&full[s], kStageBytes);
                tma_load_4d(st, &tmK, 0, slot, kvh, b, &full[s]);
                tma_load_4d(st + kBoxBytes, &tmK, 64, slot, kvh, b, &full[s]);
                tma_load_4d(st + 2 * kBoxBytes, &tmV, 0, slot, kvh, b, &full[s]);
                tma_load_4d(st + 3 * kBoxBytes, &tmV, 64, slot, kvh, b, &full[s]);
            }
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    const int qr = lane >> 2, qc = (lane & 3) * 2;
    int rows[2], nodes[2];
    bool rvalid[2];
    uint32_t anc[2][4];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int r = warp * 16 + qr + hh * 8;
        rows[hh] = r;
        rvalid[hh] = r < R;
        const int rr = row0 + (rvalid[hh] ? r : 0);
        nodes[hh] = rr / p.G;
#pragma unroll
        for (int w = 0; w < 4; ++w) anc[hh][w] = rvalid[hh] ? p.anc[nodes[hh] * 4 + w] : 0u;
    }
    // Q fragments for 8 k-steps of 16 dims
    uint32_t qa[8][4];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int rr = row0 + rows[hh];
        const __nv_bfloat16* qrow =
            p.q + (((int64_t)b * p.N + rr / p.G) * p.Hq + kvh * p.G + rr % p.G) * kD;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            uint32_t lo = 0, hi = 0;
            if (rvalid[hh]) {
                lo = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + qc);
                hi = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + qc);
            }
            qa[ks][hh] = lo;
            qa[ks][2 + hh] = hi;
        }
    }
    float o[16][4];
#pragma unroll
    for (int t = 0; t < 16; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.0f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
    bool ok = true;

    for (int i = 0; i < nmine; ++i) {
        const int s = i % kStages;
        if (!mbar_wait(&full[s], (i / kStages) & 1)) {
            atomicCAS(&g_fg_error_word, 0, FG_ETIMEOUT);
            ok = false;
            break;
        }
        const uint8_t* Ks = smem + s * kStageBytes;
        const uint8_t* Vs = Ks + 2 * kBoxBytes;
        const uint32_t ks_base = smem_u32(Ks), vs_base = smem_u32(Vs);
        float sc[8][4];
#pragma unroll
        for (int t = 0; t < 8; ++t) sc[t][0] = sc[t][1] = sc[t][2] = sc[t][3] = 0.0f;
        // S = Q K^T
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            const int box = ks >> 2;
#pragma unroll
            for (int pr = 0; pr < 4; ++pr) {
                const int m = lane >> 3;
                const int slot = (pr * 2 + (m >> 1)) * 8 + (lane & 7);
                const int col = (ks & 3) * 2 + (m & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(ks_base + box * kBoxBytes + swz(slot, col), b0, b1, b2, b3);
                mma_bf16(sc[pr * 2], qa[ks], b0, b1);
                mma_bf16(sc[pr * 2 + 1], qa[ks], b2, b3);
            }
        }
        // mask (only chunks reaching past the prefix), scale, online softmax
        const int base = (c_begin + i) * kBlockN;
        float mloc[2] = {-INFINITY, -INFINITY};
        if (base + kBlockN <= kv_len) {
#pragma unroll
            for (int t = 0; t < 8; ++t)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float v = sc[t][e] * p.scale_log2;
                    sc[t][e] = v;
                    mloc[e >> 1] = fmaxf(mloc[e >> 1], v);
                }
        } else {
#pragma unroll
            for (int t = 0; t < 8; ++t)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int hh = e >> 1;
                    const int pos = base + t * 8 + qc + (e & 1);
                    const int j = pos - kv_len;
                    const bool vis = pos < kv_len ||
                                     (pos < T && anc_bit(anc[hh][0], anc[hh][1], anc[hh][2], anc[hh][3], j));
                    const float v = vis ? sc[t][e] * p.scale_log2 : -INFINITY;
                    sc[t][e] = v;
                    mloc[hh] = fmaxf(mloc[hh], v);
                }
        }
        float alpha[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            mloc[hh] = fmaxf(mloc[hh], __shfl_xor_sync(0xffffffffu, mloc[hh], 1));
            mloc[hh] = fmaxf(mloc[hh], __shfl_xor_sync(0xffffffffu, mloc[hh], 2));
            const float mn = fmaxf(m_run[hh], mloc[hh]);
            alpha[hh] = (mn == -INFINITY) ? 1.0f : exp2f(m_run[hh] - mn);
            m_run[hh] = mn;
        }
        float rs[2] = {0.0f, 0.0f};
        uint32_t pa[4][4];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int hh = e >> 1;
                const float pv = (m_run[hh] == -INFINITY) ? 0.0f : exp2f(sc[t][e] - m_run[hh]);
                sc[t][e] = pv;
                rs[hh] += pv;
            }
            pa[t >> 1][(t & 1) * 2 + 0] = pack_bf16(sc[t][0], sc[t][1]);
            pa[t >> 1][(t & 1) * 2 + 1] = pack_bf16(sc[t][2], sc[t][3]);
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            rs[hh] += __shfl_xor_sync(0xffffffffu, rs[hh], 1);
            rs[hh] += __shfl_xor_sync(0xffffffffu, rs[hh], 2);
            l_run[hh] = l_run[hh] * alpha[hh] + rs[hh];
        }
#pragma unroll
        for (int t = 0; t < 16; ++t) {
            o[t][0] *= alpha[0];
            o[t][1] *= alpha[0];
            o[t][2] *= alpha[1];
            o[t][3] *= alpha[1];
        }
        // O += P V.  pa[kk] = {rows lo k-lo, rows hi k-lo, rows lo k-hi, rows hi k-hi}
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint32_t a[4] = {pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3]};
#pragma unroll
            for (int dp = 0; dp < 8; ++dp) {
                const int m = lane >> 3;
                const int slot = kk * 16 + (m & 1) * 8 + (lane & 7);
                const int dt = dp * 2 + (m >> 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vs_base + (dt >> 3) * kBoxBytes + swz(slot, dt & 7), b0, b1, b2, b3);
                mma_bf16(o[dp * 2], a, b0, b1);
                mma_bf16(o[dp * 2 + 1], a, b2, b3);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!ok) return;

    const int nthreads = WM * 32;
    if (p.splits == 1) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            if (!rvalid[hh]) continue;
            const int rr = row0 + rows[hh];
            __nv_bfloat16* orow = p.out + (((int64_t)b * p.N + rr / p.G) * p.Hq + kvh * p.G + rr % p.G) * kD;
            const float inv = l_run[hh] > 0.0f ? 1.0f / l_run[hh] : 0.0f;
#pragma unroll
            for (int t = 0; t < 16; ++t)
                *reinterpret_cast<__nv_bfloat162*>(orow + t * 8 + qc) =
                    __floats2bfloat162_rn(o[t][hh * 2] * inv, o[t][hh * 2 + 1] * inv);
        }
        return;
    }
    // split partials
    float* wo = p.ws_o + ((int64_t)item * p.splits + split) * (kMaxRows * kD);
    float* wml = p.ws_ml + ((int64_t)item * p.splits + split) * (2 * kMaxRows);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int r = rows[hh];
        if (!rvalid[hh]) continue;
#pragma unroll
        for (int t = 0; t < 16; ++t)
            *reinterpret_cast<float2*>(wo + r * kD + t * 8 + qc) = make_float2(o[t][hh * 2], o[t][hh * 2 + 1]);
        if ((lane & 3) == 0) {
            wml[r] = m_run[hh];
            wml[kMaxRows + r] = l_run[hh];
        }
    }
    __threadfence();
    named_sync(1, nthreads);
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(&p.ws_cnt[item], 1);
        *flag = (prev == p.splits - 1) ? 1 : 0;
    }
    named_sync(1, nthreads);
    if (*flag == 0) return;
    __threadfence();
    // merge all splits of this item
    const float* wo_all = p.ws_o + (int64_t)item * p.splits * (kMaxRows * kD);
    const float* wml_all = p.ws_ml + (int64_t)item * p.splits * (2 * kMaxRows);
    for (int e = threadIdx.x; e < R * (kD / 2); e += nthreads) {
        const int r = e / (kD / 2), d = (e % (kD / 2)) * 2;
        float mt = -INFINITY;
        for (int s2 = 0; s2 < p.splits; ++s2) mt = fmaxf(mt, __ldcg(wml_all + s2 * 2 * kMaxRows + r));
        float lt = 0.0f, a0 = 0.0f, a1 = 0.0f;
        if (mt != -INFINITY) {
            for (int s2 = 0; s2 < p.splits; ++s2) {
                const float ms = __ldcg(wml_all + s2 * 2 * kMaxRows + r);
                if (ms == -INFINITY) continue;
                const float w = exp2f(ms - mt);
                lt += w * __ldcg(wml_all + s2 * 2 * kMaxRows + kMaxRows + r);
                const float2 ov = __ldcg(reinterpret_cast<const float2*>(wo_all + (int64_t)s2 * kMaxRows * kD + r * kD + d));
                a0 += w * ov.x;
                a1 += w * ov.y;
            }
        }
        const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
        const int rr = row0 + r;
        __nv_bfloat16* orow = p.out + (((int64_t)b * p.N + rr / p.G) * p.Hq + kvh * p.G + rr % p.G) * kD;
        *reinterpret_cast<__nv_bfloat162*>(orow + d) = __floats2bfloat162_rn(a0 * inv, a1 * inv);
    }
    if (threadIdx.x == 0) p.ws_cnt[item] = 0;
}

// ------------------------------------------------------------------- f32
__global__ void tree_attn_f32_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                     const float* __restrict__ vc, int64_t sb, int64_t sh, int64_t ss,
                                     const int32_t* __restrict__ kv_len, const uint32_t* __restrict__ anc, int32_t N,
                                     int32_t Hq, int32_t Hkv, int32_t D, float scale, float* __restrict__ out) {
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
    const float* kb = kc + (int64_t)b * sb + (int64_t)kvh * sh;
    const float* vb = vc + (int64_t)b * sb + (int64_t)kvh * sh;
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

// 4-D map over [B, Hkv, capacity, D] bf16 with 64 x 64 boxes, 128B swizzle.
static bool make_kv_map(CUtensorMap* map, void* base, int32_t B, int32_t Hkv, int32_t cap, int64_t sb, int64_t sh,
                        int64_t ss) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)cap, (cuuint64_t)Hkv, (cuuint64_t)B};
    const cuuint64_t strides[3] = {(cuuint64_t)ss * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
    const cuuint32_t box[4] = {64, (cuuint32_t)kBlockN, 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int auto_splits(int32_t items, int32_t max_kv_len, int32_t n_nodes) {
    const int chunks = (max_kv_len + n_nodes + kBlockN - 1) / kBlockN;
    const int slots = 148;  // one tensor-core CTA per SM (~194 KB of shared memory each)
    int s = slots / max(1, items);
    s = max(1, min(s, chunks / 2));
    return min(s, 64);
}

}  // namespace fg

using namespace fg;

static int resolve_splits(int32_t B, int32_t n_nodes, int32_t n_q_heads, int32_t n_kv_heads, int32_t num_splits,
                          int32_t max_kv_len) {
    const int G = n_q_heads / n_kv_heads;
    const int groups = (n_nodes * G + kMaxRows - 1) / kMaxRows;
    const int items = B * n_kv_heads * groups;
    return num_splits > 0 ? num_splits : auto_splits(items, max_kv_len, n_nodes);
}

extern "C" size_t fg_tree_attention_workspace_size(int32_t B, int32_t n_nodes, int32_t n_q_heads, int32_t n_kv_heads,
                                                   int32_t head_dim, int32_t num_splits, int32_t max_kv_len) {
    if (B <= 0 || n_nodes <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads || max_kv_len < 0) return 0;
    (void)head_dim;
    const int G = n_q_heads / n_kv_heads;
    const int groups = (n_nodes * G + kMaxRows - 1) / kMaxRows;
    const size_t items = (size_t)B * n_kv_heads * groups;
    const int splits = resolve_splits(B, n_nodes, n_q_heads, n_kv_heads, num_splits, max_kv_len);
    if (splits <= 1) return 0;
    return items * splits * (size_t)(kMaxRows * kD + 2 * kMaxRows) * sizeof(float) + items * sizeof(int32_t);
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
    cudaStream_t st = (cudaStream_t)stream;
    if (dtype == FG_DTYPE_F32) {
        const int G = n_q_heads / n_kv_heads;
        if (head_dim > 128 || G > 32) return FG_ECAPACITY;
        dim3 grid(n_nodes, n_kv_heads, B);
        tree_attn_f32_kernel<<<grid, 32 * G, 0, st>>>((const float*)q, (const float*)kv->k, (const float*)kv->v,
                                                      kv->stride_b, kv->stride_h, kv->stride_s, kv_len, anc_bits,
                                                      n_nodes, n_q_heads, n_kv_heads, head_dim, scale, (float*)out);
        return launch_status();
    }
    if (dtype != FG_DTYPE_BF16) return FG_EUNSUPPORTED;
    if (head_dim != kD) return FG_EUNSUPPORTED;
    if (((uintptr_t)kv->k % 16) || ((uintptr_t)kv->v % 16) || ((kv->stride_s * 2) % 16) || ((kv->stride_h * 2) % 16) ||
        ((kv->stride_b * 2) % 16) || ((uintptr_t)q % 16) || ((uintptr_t)out % 16))
        return FG_EINVAL;
    const int G = n_q_heads / n_kv_heads;
    AttnParams p;
    p.q = (const __nv_bfloat16*)q;
    p.out = (__nv_bfloat16*)out;
    p.kv_len = kv_len;
    p.anc = anc_bits;
    p.N = n_nodes;
    p.Hq = n_q_heads;
    p.Hkv = n_kv_heads;
    p.G = G;
    p.rows_total = n_nodes * G;
    p.groups = (p.rows_total + kMaxRows - 1) / kMaxRows;
    const int items = B * n_kv_heads * p.groups;
    p.splits = resolve_splits(B, n_nodes, n_q_heads, n_kv_heads, num_splits,
                              max_kv_len > 0 ? max_kv_len : kv->capacity);
    p.scale_log2 = scale * 1.4426950408889634f;
    p.ws_o = nullptr;
    p.ws_ml = nullptr;
    p.ws_cnt = nullptr;
    if (p.splits > 1) {
        const size_t need = (size_t)items * p.splits * (kMaxRows * kD + 2 * kMaxRows) * sizeof(float) +
                            (size_t)items * sizeof(int32_t);
        if (!workspace || workspace_bytes < need || ((uintptr_t)workspace % 16)) return FG_ECAPACITY;
        p.ws_o = (float*)workspace;
        p.ws_ml = p.ws_o + (size_t)items * p.splits * kMaxRows * kD;
        p.ws_cnt = (int32_t*)(p.ws_ml + (size_t)items * p.splits * 2 * kMaxRows);
    }
    CUtensorMap mk, mv;
    if (!make_kv_map(&mk, kv->k, B, n_kv_heads, kv->capacity, kv->stride_b, kv->stride_h, kv->stride_s) ||
        !make_kv_map(&mv, kv->v, B, n_kv_heads, kv->capacity, kv->stride_b, kv->stride_h, kv->stride_s))
        return FG_EINVAL;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(tc::attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             tc::kSmemBytes);
        if (e != cudaSuccess) {
            set_cuda_error(e);
            return FG_ECUDA;
        }
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    tc::Params tp;
    tp.q = p.q;
    tp.out = p.out;
    tp.kv_len = p.kv_len;
    tp.anc = p.anc;
    tp.N = p.N;
    tp.Hq = p.Hq;
    tp.Hkv = p.Hkv;
    tp.G = p.G;
    tp.groups = p.groups;
    tp.splits = p.splits;
    tp.rows_total = p.rows_total;
    tp.scale_log2 = p.scale_log2;
    tp.ws_o = p.ws_o;
    tp.ws_ml = p.ws_ml;
    tp.ws_cnt = p.ws_cnt;
    dim3 grid(p.splits, n_kv_heads * p.groups, B);
    tc::attn_tc_kernel<<<grid, tc::kThreads, tc::kSmemBytes, st>>>(mk, mv, tp);
    return launch_status();
}

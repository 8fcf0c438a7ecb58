// fg_attention_tc.cu -- K3 on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same contract as the bf16 path of fg_tree_attention (flash-decoding GQA
// attention of one layer's tree queries over each row's KV slots, tree mask
// from ancestor bits), organised for sm_100a:
//
//   warp 0       TMA producer: K and V tiles of 128 slots x 128 dims (two
//                128x64 boxes each, 128-byte swizzle) into a 2-stage ring
//                whose K and V halves are released separately (K(i) after
//                QK(i), V(i) after PV(i)).
//   warp 1       allocates 512 TMEM columns; one elected thread issues
//                tcgen05.mma: S = Q K^T (M=128 query rows, N=128 slots,
//                K=128 dims) and O += P V (M=128, N=128 dims, K=128 slots);
//                completion is signalled with tcgen05.commit on mbarriers.
//   warps 4-7    softmax warpgroup 0: even KV tiles,
//   warps 8-11   softmax warpgroup 1: odd KV tiles.  Each warpgroup is an
//                independent online softmax with its own TMEM S tile
//                (128 columns), its own P tile in 128B-swizzled smem and its
//                own TMEM O accumulator (128 columns): one thread per query
//                row (TMEM lane = row) loads S with tcgen05.ld, applies the
//                tree mask, works in the log2 domain with lazy rescaling (O is
//                rescaled only when the row maximum grows by more than 8, so P
//                stays below 2^8) and writes P as bf16.  At the end the two
//                (m, l, O) states are merged through shared memory; each
//                warpgroup writes half of the head dimension (normalised
//                output, or fp32 partials merged by the last split).
//
// Query rows are (node, head-of-group) pairs, row = node * G + g, up to 128
// per CTA; the Q tile is loaded once by the softmax warpgroups.  The last
// tile of a row reads KV slots past the row's tree tail (up to the next
// multiple of 128, zero-filled beyond capacity): they are masked out of the
// softmax but pass through P V with weight 0, so they must hold finite
// values (a zero-initialised cache does).  Every
// mbarrier wait is bounded (about one second); on a timeout the kernel
// records FG_ETIMEOUT, stops issuing work, drains what it issued and frees
// TMEM.
#include "fg_common.cuh"

namespace fg {
namespace tc {

constexpr int kD = 128;
constexpr int kBlk = 128;                     // KV slots per tile / stage
constexpr int kStages = 2;
constexpr int kRows = 128;                    // query rows per CTA (MMA M)
constexpr int kThreads = 384;                 // 12 warps
constexpr int kQBytes = kRows * kD * 2;       // 32 KB, two 16 KB d-halves
constexpr int kPBytes = kRows * kBlk * 2;     // 32 KB per P buffer, two 16 KB slot-halves
constexpr int kBox = kBlk * 64 * 2;           // 16 KB: 128 slots x 64 dims
constexpr int kStageBytes = 4 * kBox;         // K lo/hi + V lo/hi = 64 KB
constexpr int kOffQ = 0;
constexpr int kOffP = kQBytes;                              // 32 KB
constexpr int kOffStage = kOffP + 2 * kPBytes;              // 96 KB
constexpr int kOffBar = kOffStage + kStages * kStageBytes;  // 224 KB
// The epilogue's m/l exchange of warpgroup w lives in its own P buffer,
// which no MMA reads once w's last PV has completed.  (The Q tile is not
// free at that point: the issuer may still have a QK of the other
// warpgroup's last tile outstanding.)
constexpr int kSmemBytes = kOffBar + 256 + 1024;
constexpr uint32_t kTmemCols = 512;           // S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512)
constexpr uint32_t kColO0 = 256;
constexpr int64_t kWaitNs = 1000000000LL;
constexpr float kRescaleLog2 = 8.0f;
constexpr int kMaxSplits = 128;               // the merge keeps [2 x splits x 128] floats in smem
static_assert(2 * kMaxSplits * kRows * 4 <= kOffBar, "split (m, l) tables fit below the barriers");

struct Params {
    const __nv_bfloat16* q;
    __nv_bfloat16* out;
    const int32_t* kv_len;
    const uint32_t* anc;
    int32_t N, Hq, Hkv, G, groups, splits, rows_total;
    float scale_log2;
    float* ws_o;
    float* ws_ml;
    int32_t* ws_cnt;
    const int32_t* kv_rows;  // call row -> cache row (NULL = identity)
    int32_t kv_batch;
};

// ---------------------------------------------------------------- PTX glue
__device__ __forceinline__ uint32_t sa(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ uint64_t gtime() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(b)) : "memory");
}
__device__ __forceinline__ void bar_expect(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(sa(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Non-blocking probe of a phase (never suspends the thread): the MMA issuer
// polls several barriers in turn with it.
__device__ __forceinline__ bool bar_test(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(sa(b)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: false after ~1 s or when another role aborted the CTA.
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag) {
    for (int i = 0; i < 2048; ++i)
        if (bar_try(b, parity)) return true;
    const uint64_t t0 = gtime();
    for (uint32_t i = 0;; ++i) {
        if (bar_try(b, parity)) return true;
        if ((i & 255u) == 0u) {
            if (*abort_flag) return false;
            if ((int64_t)(gtime() - t0) > kWaitNs) {
                *abort_flag = 1;
                atomicCAS(&g_fg_error_word, 0, FG_ETIMEOUT);
                return false;
            }
        }
    }
}

// Time-bounded wait that ignores the abort flag: used to drain work this
// thread already issued (TMA loads, MMAs) before TMEM or smem is released.
__device__ __forceinline__ bool bar_drain(uint64_t* b, uint32_t parity) {
    const uint64_t t0 = gtime();
    for (uint32_t i = 0;; ++i) {
        if (bar_try(b, parity)) return true;
        if ((i & 255u) == 0u && (int64_t)(gtime() - t0) > kWaitNs) {
            atomicCAS(&g_fg_error_word, 0, FG_ETIMEOUT);
            return false;
        }
    }
}

__device__ __forceinline__ void tma_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, uint64_t* b) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(sa(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(sa(b))
        : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2, version 1).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, M = 128.
__host__ __device__ constexpr uint32_t idesc_bf16(int n, bool b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(kRows >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa(b))
                 : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 128 consecutive fp32 columns of this thread's TMEM lane; the wait sits in
// the same asm statement so no use of the registers can precede it.
__device__ __forceinline__ void tld128(uint32_t taddr, float* v) {
    uint32_t r[128];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, %96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, %112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%128];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]),
          "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]),
          "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]),
          "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]),
          "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]),
          "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]),
          "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]),
          "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]),
          "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 128; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tst32(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// Visibility of the 32 KV slots p0 .. p0 + 31 for one query row: bit t set
// when slot p0 + t is a prefix slot (< kv_len) or a tree slot (< T) whose
// tree index p0 + t - kv_len is an ancestor-or-self bit of (a0, a1, a2, a3).
// Branch-free: funnel shifts over the 128-bit ancestor mask.
__device__ __forceinline__ uint32_t visible_bits(int p0, int kv_len, int T, uint32_t a0, uint32_t a1, uint32_t a2,
                                                 uint32_t a3) {
    const int np = min(max(kv_len - p0, 0), 32);
    const uint32_t prefix = np >= 32 ? 0xffffffffu : ((1u << np) - 1u);
    const int nt = min(max(T - p0, 0), 32);
    const uint32_t live = nt >= 32 ? 0xffffffffu : ((1u << nt) - 1u);
    const int j0 = p0 - kv_len;  // tree index of bit 0, may be negative
    uint32_t tree;
    if (j0 < 0) {
        tree = j0 > -32 ? (a0 << (-j0)) : 0u;
    } else {
        const int q = j0 >> 5, sh = j0 & 31;
        const uint32_t lo = q == 0 ? a0 : q == 1 ? a1 : q == 2 ? a2 : q == 3 ? a3 : 0u;
        const uint32_t hi = q == 0 ? a1 : q == 1 ? a2 : q == 2 ? a3 : 0u;
        tree = __funnelshift_r(lo, hi, sh);
    }
    return (prefix | tree) & live;
}

// Byte offset of 16-byte column c of row r in a 128B-swizzled tile of 128-byte rows.
__device__ __forceinline__ uint32_t sw128(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }


__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

struct Bars {
    uint64_t k_full[kStages];
    uint64_t k_empty[kStages];
    uint64_t v_full[kStages];
    uint64_t v_empty[kStages];
    uint64_t s_full[2];
    uint64_t s_free[2];
    uint64_t p_full[2];
    uint64_t o_done[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort_flag;
    int last_flag;
};

__global__ void __launch_bounds__(kThreads, 1) attn_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                                                              const __grid_constant__ CUtensorMap tmV, Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
    volatile int* abort_flag = &bars->abort_flag;

    const int split = blockIdx.x;
    const int kvh = blockIdx.y / p.groups, grp = blockIdx.y % p.groups;
    const int b = blockIdx.z;
    // cache row of this call row (a row outside the cache records FG_EINVAL
    // and reads row 0, so the loads stay in bounds)
    const int bkv = max(cache_row(p.kv_rows, p.kv_batch, b), 0);
    const int row0 = grp * kRows;
    const int R = min(kRows, p.rows_total - row0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kv_len = p.kv_len[b];
    const int T = kv_len + p.N;
    const int nblk = (T + kBlk - 1) / kBlk;
    const int per = (nblk + p.splits - 1) / p.splits;
    const int c0 = min(nblk, split * per);
    const int nmine = min(nblk, c0 + per) - c0;
    const int item = (b * p.Hkv + kvh) * p.groups + grp;

    // K(i) and V(i) go to stage i % kStages; K and V halves have their own barriers
    auto load_k = [&](int i) {
        const int s = i % kStages;
        uint8_t* st = smem + kOffStage + s * kStageBytes;
        const int slot = (c0 + i) * kBlk;
        bar_expect(&bars->k_full[s], 2 * kBox);
        tma_4d(st, &tmK, 0, slot, kvh, bkv, &bars->k_full[s]);
        tma_4d(st + kBox, &tmK, 64, slot, kvh, bkv, &bars->k_full[s]);
    };
    auto load_v = [&](int i) {
        const int s = i % kStages;
        uint8_t* st = smem + kOffStage + s * kStageBytes + 2 * kBox;
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
        for (int i = 0; i < 2; ++i) {
            bar_init(&bars->s_full[i], 1);
            bar_init(&bars->s_free[i], 4);
            bar_init(&bars->p_full[i], 4);
            bar_init(&bars->o_done[i], 1);
        }
        bar_init(&bars->drain, 1);
        bars->abort_flag = 0;
        bars->last_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // The first tiles of the ring load while Q is staged and TMEM
        // allocated.  Tiles wholly inside the prefix (written by earlier
        // rounds) may load before the preceding kernel -- the RoPE/KV write
        // of this layer, launched as our programmatic predecessor -- has
        // finished; the others wait for it below.
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
    // Q and this round's tree K/V slots are written by the preceding kernel:
    // every thread waits for it (a no-op without programmatic launch); the
    // projection after this kernel may then start fetching its weights
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0)
        for (int i = 0; i < min(kStages, nmine); ++i)
            if ((c0 + i + 1) * kBlk > kv_len) {
                load_k(i);
                load_v(i);
            }
    const int wg = warp >= 4 ? (warp - 4) >> 2 : -1;  // softmax warpgroup
    const int r = (warp & 3) * 32 + lane;              // query row = TMEM lane
    // Q tile (rows beyond R zero) -> swizzled smem; warpgroup w loads dims [64w, 64w + 64)
    if (wg >= 0) {
        uint8_t* qs = smem + kOffQ + wg * (kRows * 128);
        const bool valid = r < R;
        const int rr = row0 + (valid ? r : 0);
        const __nv_bfloat16* qrow = p.q + (((int64_t)b * p.N + rr / p.G) * p.Hq + kvh * p.G + rr % p.G) * kD + wg * 64;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint4 v = valid ? *reinterpret_cast<const uint4*>(qrow + c * 8) : make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(qs + sw128(r, c)) = v;
        }
        fence_async_smem();
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0 || warp == 2) {
        // ------------------------------------- TMA producers: K (warp 0), V (warp 2)
        // K(i) reuses the stage of K(i - 2) once QK(i - 2) has completed, V(i)
        // that of V(i - 2) once PV(i - 2) has: the two streams never wait on
        // each other, so a K load is not held up behind a PV.
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
            // the last loads of each stage have landed before this CTA's smem goes away
            for (int j = max(0, issued - kStages); j < issued; ++j) bar_drain(&full[j % kStages], (j / kStages) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        // tile i belongs to warpgroup i & 1: S tile (i & 1), P tile (i & 1), O
        // (i & 1).  QK(i) needs K(i) and S(i - 2) read; PV(i) needs V(i) and
        // P(i).  The two streams are polled without blocking and issued as
        // soon as their operands are ready, each in tile order.
        if (lane == 0) {
            constexpr uint32_t id_qk = idesc_bf16(kBlk, false);
            constexpr uint32_t id_pv = idesc_bf16(kD, true);
            const uint32_t q_addr = sa(smem + kOffQ);
            int nq = 0, npv = 0;
            uint64_t t_idle = 0;
            for (uint32_t spin = 0; npv < nmine; ++spin) {
                bool progress = false;
                if (nq < nmine && bar_test(&bars->k_full[nq % kStages], (nq / kStages) & 1) &&
                    (nq < 2 || bar_test(&bars->s_free[nq & 1], ((nq >> 1) - 1) & 1))) {
                    fence_after();
                    const uint32_t k_addr = sa(smem + kOffStage + (nq % kStages) * kStageBytes);
#pragma unroll
                    for (int kk = 0; kk < kD / 16; ++kk) {
                        const uint64_t da = sdesc(q_addr + (kk >> 2) * (kRows * 128) + (kk & 3) * 32, 16, 1024);
                        const uint64_t db = sdesc(k_addr + (kk >> 2) * kBox + (kk & 3) * 32, 16, 1024);
                        umma(tmem + (uint32_t)((nq & 1) * kBlk), da, db, id_qk, kk > 0 ? 1u : 0u);
                    }
                    umma_commit(&bars->s_full[nq & 1]);
                    umma_commit(&bars->k_empty[nq % kStages]);
                    ++nq;
                    progress = true;
                }
                if (npv < nq && bar_test(&bars->v_full[npv % kStages], (npv / kStages) & 1) &&
                    bar_test(&bars->p_full[npv & 1], (npv >> 1) & 1)) {
                    fence_after();
                    const uint32_t p_addr = sa(smem + kOffP + (npv & 1) * kPBytes);
                    const uint32_t v_addr = sa(smem + kOffStage + (npv % kStages) * kStageBytes + 2 * kBox);
                    const uint32_t o_col = kColO0 + (uint32_t)(npv & 1) * kD;
#pragma unroll
                    for (int kk = 0; kk < kBlk / 16; ++kk) {
                        const uint64_t da = sdesc(p_addr + (kk >> 2) * (kRows * 128) + (kk & 3) * 32, 16, 1024);
                        const uint64_t db = sdesc(v_addr + kk * 2048, kBox, 1024);
                        umma(tmem + o_col, da, db, id_pv, (npv >= 2 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(&bars->o_done[npv & 1]);
                    umma_commit(&bars->v_empty[npv % kStages]);
                    ++npv;
                    progress = true;
                }
                if (progress) {
                    t_idle = 0;
                } else if ((spin & 255u) == 0u) {
                    // bounded like every other wait: ~1 s without progress aborts the CTA
                    if (*abort_flag) break;
                    const uint64_t now = gtime();
                    if (t_idle == 0) {
                        t_idle = now;
                    } else if ((int64_t)(now - t_idle) > kWaitNs) {
                        *abort_flag = 1;
                        atomicCAS(&g_fg_error_word, 0, FG_ETIMEOUT);
                        break;
                    }
                }
            }
            // everything issued has completed before TMEM is read or freed
            umma_commit(&bars->drain);
            bar_drain(&bars->drain, 0);
        }
    } else if (wg >= 0) {
        // ------------------------------------------- softmax warpgroup wg
        const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t s_col = (uint32_t)(wg * kBlk);
        const uint32_t o_col = kColO0 + (uint32_t)wg * kD;
        const bool valid = r < R;
        const int rr = row0 + (valid ? r : 0);
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
        const int n_own = (nmine - wg + 1) / 2;  // tiles wg, wg + 2, ...
        // Every tcgen05.ld / tcgen05.st below is a warp-collective
        // (.sync.aligned) instruction: control flow around them is kept
        // warp-uniform (__all_sync / __any_sync), per-row choices are selects.
        constexpr unsigned kFull = 0xffffffffu;
        for (int j = 0; j < n_own; ++j) {
            const int i = 2 * j + wg;
            if (!__all_sync(kFull, bar_wait(&bars->s_full[wg], j & 1, abort_flag))) {
                ok = false;
                break;
            }
            fence_after();
            float sv[kBlk];
            static_assert(kBlk == 128, "S tile is read with one 128-column TMEM load");
            tld128(tmem + lane_addr + s_col, sv);
            fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&bars->s_free[wg]);
            // tree mask (last tiles only), then the raw row maximum; the
            // scale (> 0) is applied inside the exponent
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
            const float mx = fmaxf(fmaxf(mq0, mq1), fmaxf(mq2, mq3)) * p.scale_log2;  // -inf stays -inf
            // previous PV of this warpgroup done: P tile free and O stable
            if (j >= 1 && !__all_sync(kFull, bar_wait(&bars->o_done[wg], (j - 1) & 1, abort_flag))) {
                ok = false;
                break;
            }
            const bool grow = mx > m_used + kRescaleLog2 || (m_used == -INFINITY && mx != -INFINITY);
            const float alpha = grow ? ((m_used == -INFINITY) ? 0.0f : ex2(m_used - mx)) : 1.0f;
            const bool rescale_o = j >= 1 && __any_sync(kFull, grow);
            if (grow) {
                l *= alpha;
                m_used = mx;
            }
            // P = exp2(s - m_used) -> bf16, swizzled rows of 128 bytes
            uint8_t* pbuf = smem + kOffP + wg * kPBytes;
            const float mneg = m_used == -INFINITY ? 0.0f : -m_used;
            float rs0 = 0.0f, rs1 = 0.0f;
#pragma unroll
            for (int c = 0; c < kBlk / 8; ++c) {
                float e[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) e[q] = ex2(fmaf(sv[c * 8 + q], p.scale_log2, mneg));  // ex2(-inf) = 0
                const float part = ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
                if (c & 1) rs1 += part; else rs0 += part;
                uint4 w;
                w.x = pack2(e[0], e[1]);
                w.y = pack2(e[2], e[3]);
                w.z = pack2(e[4], e[5]);
                w.w = pack2(e[6], e[7]);
                // slot-halves of 64 slots, each a 128B-swizzled 128 x 128-byte tile
                *reinterpret_cast<uint4*>(pbuf + (c >> 3) * (kRows * 128) + sw128(r, c & 7)) = w;
            }
            l += rs0 + rs1;
            if (rescale_o) {
                // O holds this warpgroup's PV up to its previous tile: rescale
                // in TMEM (after the S values are dead, to keep them in registers)
                fence_after();
#pragma unroll 1
                for (int cch = 0; cch < kD; cch += 32) {
                    float ov[32];
                    tld32(tmem + lane_addr + o_col + cch, ov);
#pragma unroll
                    for (int c = 0; c < 32; ++c) ov[c] *= alpha;
                    tst32(tmem + lane_addr + o_col + cch, ov);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            }
            fence_async_smem();
            fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&bars->p_full[wg]);
        }
        // ---- epilogue: last PV of this warpgroup, then merge the two states
        if (ok && n_own > 0) ok = __all_sync(kFull, bar_wait(&bars->o_done[wg], (n_own - 1) & 1, abort_flag));
        fence_after();
        // Each warpgroup publishes (m, l) in its own P buffer, dead once its
        // last PV has completed.  A warpgroup without tiles writes nothing:
        // its state (m = -inf, l = 0) is implied by the CTA-uniform tile
        // counts.  (After an abort a PV may still read the buffer; the CTA
        // then writes no output.)
        const int n0 = (nmine + 1) / 2, n1 = nmine / 2;
        if (n_own > 0) {
            float* mine = reinterpret_cast<float*>(smem + kOffP + wg * kPBytes);  // [m | l] x 128 rows
            mine[r] = ok ? m_used : -INFINITY;
            mine[kRows + r] = ok ? l : 0.0f;
        }
        // both O accumulators are final once both warpgroups pass this barrier
        fence_before();
        asm volatile("bar.sync 2, 256;" ::: "memory");
        fence_after();
        const float* x0 = reinterpret_cast<const float*>(smem + kOffP);
        const float* x1 = reinterpret_cast<const float*>(smem + kOffP + kPBytes);
        const float m0 = n0 > 0 ? x0[r] : -INFINITY, l0 = n0 > 0 ? x0[kRows + r] : 0.0f;
        const float m1 = n1 > 0 ? x1[r] : -INFINITY, l1 = n1 > 0 ? x1[kRows + r] : 0.0f;
        const float mt = fmaxf(m0, m1);
        // a warpgroup without tiles left its O uninitialised and it is never read
        const float w0 = (m0 != -INFINITY) ? ex2(m0 - mt) : 0.0f;
        const float w1 = (m1 != -INFINITY) ? ex2(m1 - mt) : 0.0f;
        const float lt = l0 * w0 + l1 * w1;
        const int aborted = *abort_flag;
        if (__all_sync(kFull, ok) && !__any_sync(kFull, aborted != 0)) {
            // this warpgroup writes dims [64 wg, 64 wg + 64) of the merged row
            const int d0 = wg * 64;
            float* wo = nullptr;
            if (p.splits > 1) {
                wo = p.ws_o + ((int64_t)item * p.splits + split) * (kRows * kD) + (int64_t)r * kD;
                if (wg == 0) {
                    float* wml = p.ws_ml + ((int64_t)item * p.splits + split) * (2 * kRows);
                    wml[r] = (w0 > 0.0f || w1 > 0.0f) ? mt : -INFINITY;
                    wml[kRows + r] = lt;
                }
            }
            const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
            __nv_bfloat16* orow = p.out + (((int64_t)b * p.N + rr / p.G) * p.Hq + kvh * p.G + rr % p.G) * kD;
#pragma unroll 1
            for (int cch = 0; cch < 64; cch += 32) {
                float oa[32], ob[32];
                if (n0 > 0) {
                    tld32(tmem + lane_addr + kColO0 + d0 + cch, oa);
                } else {
#pragma unroll
                    for (int c = 0; c < 32; ++c) oa[c] = 0.0f;
                }
                if (n1 > 0) {
                    tld32(tmem + lane_addr + kColO0 + kD + d0 + cch, ob);
                } else {
#pragma unroll
                    for (int c = 0; c < 32; ++c) ob[c] = 0.0f;
                }
#pragma unroll
                for (int c = 0; c < 32; ++c) oa[c] = (w0 > 0.0f ? oa[c] * w0 : 0.0f) + (w1 > 0.0f ? ob[c] * w1 : 0.0f);
                if (p.splits == 1) {
                    if (valid) {
#pragma unroll
                        for (int c = 0; c < 32; c += 8) {
                            uint4 w;
                            w.x = pack2(oa[c] * inv, oa[c + 1] * inv);
                            w.y = pack2(oa[c + 2] * inv, oa[c + 3] * inv);
                            w.z = pack2(oa[c + 4] * inv, oa[c + 5] * inv);
                            w.w = pack2(oa[c + 6] * inv, oa[c + 7] * inv);
                            *reinterpret_cast<uint4*>(orow + d0 + cch + c) = w;
                        }
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < 32; c += 4)
                        *reinterpret_cast<float4*>(wo + d0 + cch + c) = make_float4(oa[c], oa[c + 1], oa[c + 2], oa[c + 3]);
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
    const float* wo_all = p.ws_o + (int64_t)item * p.splits * (kRows * kD);
    const float* wml_all = p.ws_ml + (int64_t)item * p.splits * (2 * kRows);
    // (1) every split's (m, l) per row -> shared memory in one parallel pass
    // (Q, P and the ring are idle now; splits <= kMaxSplits), then per row
    // the weight of each split, exp2(m_s - m) / l, in place of m_s
    float* wt = reinterpret_cast<float*>(smem);  // [split][row]
    float* ls = wt + p.splits * kRows;           // [split][row]
    for (int e = threadIdx.x; e < p.splits * R; e += blockDim.x) {
        const int s2 = e / R, rw = e - s2 * R;
        wt[s2 * kRows + rw] = __ldcg(wml_all + s2 * 2 * kRows + rw);
        ls[s2 * kRows + rw] = __ldcg(wml_all + s2 * 2 * kRows + kRows + rw);
    }
    __syncthreads();
    for (int rw = threadIdx.x; rw < R; rw += blockDim.x) {
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
    // (2) out[row, 4 dims] = sum_s wt[s][row] O_s[row, 4 dims]; each thread
    // keeps four such outputs in flight so that the partials' L2 reads overlap
    // (partials are finite: splits without visible slots wrote zeros)
    const int total = R * (kD / 4);
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
                const int rr = row0 + rw;
                __nv_bfloat16* orow = p.out + (((int64_t)b * p.N + rr / p.G) * p.Hq + kvh * p.G + rr % p.G) * kD;
                uint2 pk;
                pk.x = pack2(acc[u].x, acc[u].y);
                pk.y = pack2(acc[u].z, acc[u].w);
                *reinterpret_cast<uint2*>(orow + d) = pk;
            }
        }
    }
    if (threadIdx.x == 0) p.ws_cnt[item] = 0;
}

}  // namespace tc
}  // namespace fg

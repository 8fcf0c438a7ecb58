// fg_accept.cu -- K4: exact_target acceptance walk + extract_path compaction.
//
// One CTA (512 threads) per row.  The walk follows exact_accept_paths_batch
// (flashgrpo_b200/decoding/acceptance.py:183-267): at the current parent it
// draws a target token (fg-icdf-v1 over the parent's logits row), accepts the
// first child (in node order) carrying that token, otherwise returns the draw
// as the correction token and stops.  The post-accept rules of
// flash_medusa_decoder.py:2289-2343 (clip to the remaining length, EOS cut,
// pending correction only for uncut unfinished paths) follow, then the
// accepted slots are compacted in every layer (kv_extraction.py:34-84) and
// the next round's hidden state is gathered (flash_medusa_decoder.py:2829-2835).
//
// Compaction hazard: destination slot j and source slot path[j] overlap when
// path[j'] == j for an earlier j'.  Each thread owns one 16-byte column of one
// (layer, K|V, head) and loads the column of every path entry before storing
// any, so no ordering between threads is needed.
#include "fg_common.cuh"
#include "fg_sampler.cuh"
#include "fg_nucleus.cuh"

namespace fg {

struct KvPtrs {
    uint64_t k[FG_MAX_LAYERS];
    uint64_t v[FG_MAX_LAYERS];
};

struct AcceptParams {
    const void* logits;
    int64_t logits_row_stride;
    int32_t vocab;
    const int32_t* slot;
    const int32_t* tokens;
    const int32_t* parents;
    int32_t parent_stride;
    const int32_t* n_nodes;
    int32_t n_nodes_shared;
    int32_t nmax;
    const float* uniforms;
    int32_t u_stride;
    int32_t do_sample;
    float temperature;
    float top_p;
    int32_t top_k;
    int32_t eos_id;
    int32_t max_length;
    int32_t* row_len;
    int32_t update_len;
    int32_t* active;
    int32_t dcap;
    int32_t* acc_tokens;
    int32_t* acc_nodes;
    int32_t* acc_len;
    int32_t* correction;
    int32_t* pending;
    int32_t* last_node;
    int32_t* finished;
    int32_t n_layers;
    int32_t kv_elem_bytes;
    int32_t n_kv_heads;
    int32_t head_dim;
    int64_t kv_stride_b;
    int64_t kv_stride_h;
    int64_t kv_stride_s;
    const void* tree_hidden;
    void* hidden_out;
    int32_t hidden_dim;
    int32_t hidden_elem_bytes;
    const int32_t* kv_rows;  // row -> cache row for the compaction (NULL = identity)
    int32_t kv_batch;
    const int32_t* drawn;    // parallel draws per packed logits row (NULL = draw during the walk)
    int64_t* acc_total;      // += the rows' acc_len (NULL = skip)
    int32_t* round_counter;  // += 1 per call (NULL = skip)
};

// CTAs per row and threads per CTA of the clustered walk
constexpr int kAcceptCtas = 8;
constexpr int kAcceptClusterThreads = 256;

// g_fg_error_word is defined in fg_abi.cu (same translation unit).
__device__ __forceinline__ void record_error(int32_t code) { atomicCAS(&g_fg_error_word, 0, code); }

// The clustered walk's compaction: the same moves in path order, four
// entries at a time (their loads before their stores).  A walk path is
// strictly increasing (every accepted node is a child of the previous one
// and follows it in node order, which the walk checks), so path[j] >= j:
// every later source slot lies past every destination written before it,
// and only one batch of values is held in registers.
__device__ void compact_row_in_order(const KvPtrs& kv, int32_t n_layers, int32_t elem_bytes, int32_t n_heads,
                                     int32_t head_dim, int64_t sb, int64_t sh, int64_t ss, int32_t b, int32_t base,
                                     const int32_t* path, int32_t a, int32_t part, int32_t parts) {
    const int32_t cols = head_dim * elem_bytes / 16;
    const int64_t items = (int64_t)n_layers * 2 * n_heads * cols;
    for (int64_t it = (int64_t)part * blockDim.x + threadIdx.x; it < items; it += (int64_t)parts * blockDim.x) {
        const int32_t c = (int32_t)(it % cols);
        int64_t g = it / cols;
        const int32_t h = (int32_t)(g % n_heads);
        g /= n_heads;
        const int32_t which = (int32_t)(g % 2);
        const int32_t l = (int32_t)(g / 2);
        uint8_t* rowp = reinterpret_cast<uint8_t*>(which == 0 ? kv.k[l] : kv.v[l]) +
                        ((int64_t)b * sb + (int64_t)h * sh) * elem_bytes + (int64_t)c * 16;
        for (int32_t j0 = 0; j0 < a; j0 += 4) {
            uint4 vals[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int32_t j = j0 + q;
                if (j < a && path[j] != j)
                    vals[q] = *reinterpret_cast<const uint4*>(rowp + (int64_t)(base + path[j]) * ss * elem_bytes);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int32_t j = j0 + q;
                if (j < a && path[j] != j)
                    *reinterpret_cast<uint4*>(rowp + (int64_t)(base + j) * ss * elem_bytes) = vals[q];
            }
        }
    }
}

// Moves row b's accepted slots in every layer.  path[j] < FG_MAX_PATH nodes.
// The (layer, K|V, head, column) items are dealt to `parts` CTAs (part =
// this CTA's index among them); an item is one thread's alone.
__device__ void compact_row(const KvPtrs& kv, int32_t n_layers, int32_t elem_bytes, int32_t n_heads,
                            int32_t head_dim, int64_t sb, int64_t sh, int64_t ss, int32_t b, int32_t base,
                            const int32_t* path, int32_t a, int32_t part = 0, int32_t parts = 1) {
    const int32_t cols = head_dim * elem_bytes / 16;  // 16-byte columns per vector
    const int64_t items = (int64_t)n_layers * 2 * n_heads * cols;
    for (int64_t it = (int64_t)part * blockDim.x + threadIdx.x; it < items; it += (int64_t)parts * blockDim.x) {
        const int32_t c = (int32_t)(it % cols);
        int64_t g = it / cols;
        const int32_t h = (int32_t)(g % n_heads);
        g /= n_heads;
        const int32_t which = (int32_t)(g % 2);
        const int32_t l = (int32_t)(g / 2);
        uint8_t* rowp = reinterpret_cast<uint8_t*>(which == 0 ? kv.k[l] : kv.v[l]) +
                        ((int64_t)b * sb + (int64_t)h * sh) * elem_bytes + (int64_t)c * 16;
        uint4 vals[FG_MAX_PATH];
#pragma unroll
        for (int j = 0; j < FG_MAX_PATH; ++j)
            if (j < a) vals[j] = *reinterpret_cast<const uint4*>(rowp + (int64_t)(base + path[j]) * ss * elem_bytes);
#pragma unroll
        for (int j = 0; j < FG_MAX_PATH; ++j)
            if (j < a && path[j] != j) *reinterpret_cast<uint4*>(rowp + (int64_t)(base + j) * ss * elem_bytes) = vals[j];
    }
}

// S == 1: one CTA of 512 threads per row.  S > 1: a cluster of S CTAs of
// kAcceptClusterThreads threads per row, for fg-icdf-v1 draws (no nucleus,
// T > 0, no parallel draws): every CTA walks the tree redundantly on the
// same draws (cluster_sample, its e_i buffer in dynamic shared memory), CTA 0
// writes the row's outputs, the compaction and the hidden copy are dealt
// over the S CTAs, and the lengths / active flags change only after a
// cluster barrier (every CTA has read them by then).
template <typename T, int S>
__global__ void __launch_bounds__(S > 1 ? kAcceptClusterThreads : FG_SAMPLE_LANES, S > 1 ? 4 : 1)
    accept_extract_kernel(AcceptParams p, KvPtrs kv) {
    __shared__ int32_t s_child;
    __shared__ int32_t s_match;
    __shared__ int32_t s_path[FG_MAX_PATH];
    __shared__ int32_t s_tok[FG_MAX_PATH];
    __shared__ int32_t s_a, s_corr, s_err;
    const int32_t b = blockIdx.x / S;
    const int tid = threadIdx.x;
    const uint32_t rank = S > 1 ? cl_rank() : 0;
    const int32_t* tk = p.tokens + (int64_t)b * p.nmax;
    const int32_t* pa = p.parents + (int64_t)b * p.parent_stride;
    const int32_t* sl = p.slot + (int64_t)b * p.nmax;
    const int32_t n = p.n_nodes ? p.n_nodes[b] : p.n_nodes_shared;
    const bool row_active = p.active == nullptr || p.active[b] != 0;
    if (!row_active) {
        if (rank != 0) return;
        if (tid < p.dcap) {
            p.acc_tokens[(int64_t)b * p.dcap + tid] = -1;
            p.acc_nodes[(int64_t)b * p.dcap + tid] = -1;
        }
        if (tid == 0) {
            p.acc_len[b] = 0;
            p.correction[b] = -1;
            p.pending[b] = -1;
            p.last_node[b] = 0;
            p.finished[b] = 1;
            if (p.round_counter != nullptr && b == 0) atomicAdd(p.round_counter, 1);
        }
        return;
    }
    if (tid == 0) {
        s_a = 1;
        s_corr = -1;
        s_err = 0;
        s_path[0] = 0;
        s_tok[0] = tk[0];
    }
    __syncthreads();
    int32_t parent = 0;
    for (int step = 0;; ++step) {
        // first child of `parent` in node order
        if (tid == 0) s_child = 0x7fffffff;
        __syncthreads();
        for (int32_t j = 1 + tid; j < n; j += blockDim.x)
            if (pa[j] == parent) atomicMin(&s_child, j);
        __syncthreads();
        if (s_child == 0x7fffffff) break;
        if (s_a >= FG_MAX_PATH || step >= p.u_stride) {
            if (tid == 0) s_err = FG_ECAPACITY;
            __syncthreads();
            break;
        }
        const int32_t srow = sl[parent];
        if (srow < 0) {
            if (tid == 0) s_err = FG_EINVAL;
            __syncthreads();
            break;
        }
        int32_t drawn;
        if (p.drawn) {
            // drawn by draw_internal_kernel at this node with this step's uniform
            drawn = p.drawn[srow];
        } else {
            const T* row = static_cast<const T*>(p.logits) + (int64_t)srow * p.logits_row_stride;
            const float u = p.uniforms[(int64_t)b * p.u_stride + step];
            if constexpr (S == 1) {
                __shared__ SampleSmem sm;
                __shared__ NucleusSmem ns;
                drawn = sample_cuts(p.do_sample, p.temperature, p.top_p, p.top_k, p.vocab)
                            ? block_sample_kept<T>(row, p.vocab, p.temperature, p.top_p, p.top_k, u, sm, ns)
                            : block_sample<T>(row, p.vocab, p.temperature, p.do_sample != 0, u, sm);
            } else {
                __shared__ ClusterSampleSmem<S, kAcceptClusterThreads> cs;
                extern __shared__ __align__(16) float ebuf[];
                drawn = cluster_sample<T, S, kAcceptClusterThreads>(row, p.vocab, p.temperature, u, cs, ebuf);
            }
        }
        if (tid == 0) s_match = 0x7fffffff;
        __syncthreads();
        for (int32_t j = s_child + tid; j < n; j += blockDim.x)
            if (pa[j] == parent && tk[j] == drawn) atomicMin(&s_match, j);
        __syncthreads();
        const int32_t match = s_match;
        if (match == 0x7fffffff) {
            if (tid == 0) s_corr = drawn;
            __syncthreads();
            break;
        }
        if (match <= parent) {  // children follow their parent in node order
            if (tid == 0) s_err = FG_EINVAL;
            __syncthreads();
            break;
        }
        if (tid == 0) {
            s_path[s_a] = match;
            s_tok[s_a] = drawn;
            s_a += 1;
        }
        parent = match;
        __syncthreads();
    }
    if (s_err != 0) {
        if (tid == 0 && rank == 0) record_error(s_err);
        return;
    }
    // post-accept rules
    const int32_t raw = s_a;
    const int32_t len0 = p.row_len[b];
    int32_t a = raw;
    const int32_t max_accept = max(1, p.max_length - len0);
    a = min(a, max_accept);
    bool eos_seen = false;
    for (int32_t j = 0; j < a; ++j)
        if (s_tok[j] == p.eos_id) {
            a = j + 1;
            eos_seen = true;
            break;
        }
    const bool fin = eos_seen || (len0 + a >= p.max_length);
    if (rank == 0 && tid < p.dcap) {
        p.acc_tokens[(int64_t)b * p.dcap + tid] = tid < a ? s_tok[tid] : -1;
        p.acc_nodes[(int64_t)b * p.dcap + tid] = tid < a ? s_path[tid] : -1;
    }
    if (rank == 0 && tid == 0) {
        p.acc_len[b] = a;
        p.correction[b] = s_corr;
        p.pending[b] = (s_corr >= 0 && a == raw && !fin) ? s_corr : -1;
        p.last_node[b] = s_path[a - 1];
        p.finished[b] = fin ? 1 : 0;
    }
    // extract_path compaction of the accepted slots (in the row's cache row)
    const int32_t bk = cache_row(p.kv_rows, p.kv_batch, b);
    if (p.n_layers > 0 && bk >= 0) {
        if constexpr (S > 1)
            compact_row_in_order(kv, p.n_layers, p.kv_elem_bytes, p.n_kv_heads, p.head_dim, p.kv_stride_b,
                                 p.kv_stride_h, p.kv_stride_s, bk, len0, s_path, a, (int32_t)rank, S);
        else
            compact_row(kv, p.n_layers, p.kv_elem_bytes, p.n_kv_heads, p.head_dim, p.kv_stride_b, p.kv_stride_h,
                        p.kv_stride_s, bk, len0, s_path, a);
    }
    // next-round hidden state
    if (p.hidden_out != nullptr) {
        const int64_t bytes = (int64_t)p.hidden_dim * p.hidden_elem_bytes;
        const uint8_t* src = static_cast<const uint8_t*>(p.tree_hidden) + ((int64_t)b * p.nmax + s_path[a - 1]) * bytes;
        uint8_t* dst = static_cast<uint8_t*>(p.hidden_out) + (int64_t)b * bytes;
        for (int64_t o = ((int64_t)rank * blockDim.x + tid) * 16; o < bytes; o += (int64_t)S * blockDim.x * 16)
            *reinterpret_cast<uint4*>(dst + o) = *reinterpret_cast<const uint4*>(src + o);
    }
    if constexpr (S > 1)
        cl_sync();
    else
        __syncthreads();
    if (rank == 0 && tid == 0) {
        if (p.update_len) p.row_len[b] = len0 + a;
        if (fin && p.active != nullptr) p.active[b] = 0;
        if (p.acc_total != nullptr) atomicAdd(reinterpret_cast<unsigned long long*>(p.acc_total), (unsigned long long)a);
        if (p.round_counter != nullptr && b == 0) atomicAdd(p.round_counter, 1);
    }
}

// The walk's target draws, all at once: the draw at internal node n of row b
// uses logits row slot[b][n] and uniform u[b][depth(n) - 1] -- the step at
// which the walk stands on n -- so every internal node's draw is fixed
// before the walk and they run in parallel, one CTA per packed logits row
// (row j = b * n_int + rank, node internal[rank]; n_int from the tree's plan
// on the device when plan_out is set).  The walk then only reads them.
template <typename T>
__global__ void __launch_bounds__(FG_SAMPLE_LANES) draw_internal_kernel(AcceptParams p, int32_t B,
                                                                        const int32_t* internal, const int32_t* depths,
                                                                        const int32_t* plan_out, int32_t n_int_static,
                                                                        int32_t* drawn) {
    __shared__ SampleSmem sm;
    __shared__ NucleusSmem ns;
    const int32_t n_int = plan_out ? plan_out[11] : n_int_static;
    const int32_t j = blockIdx.x;
    if (n_int <= 0 || j >= B * n_int) return;
    const int32_t b = j / n_int, rank = j - b * n_int;
    const int32_t node = internal[rank];
    if (p.active != nullptr && p.active[b] == 0) {
        if (threadIdx.x == 0) drawn[j] = -1;
        return;
    }
    const int32_t step = depths[node] - 1;
    if (node < 0 || node >= p.nmax || p.slot[(int64_t)b * p.nmax + node] != j || step < 0 || step >= p.u_stride) {
        if (threadIdx.x == 0) {
            drawn[j] = -1;
            record_error(FG_EINVAL);
        }
        return;
    }
    const T* row = static_cast<const T*>(p.logits) + (int64_t)j * p.logits_row_stride;
    const float u = p.uniforms[(int64_t)b * p.u_stride + step];
    const int32_t t = sample_cuts(p.do_sample, p.temperature, p.top_p, p.top_k, p.vocab)
                          ? block_sample_kept<T>(row, p.vocab, p.temperature, p.top_p, p.top_k, u, sm, ns)
                          : block_sample<T>(row, p.vocab, p.temperature, p.do_sample != 0, u, sm);
    if (threadIdx.x == 0) drawn[j] = t;
}

__global__ void extract_path_kernel(KvPtrs kv, int32_t n_layers, int32_t elem_bytes, int32_t n_heads,
                                    int32_t head_dim, int64_t sb, int64_t sh, int64_t ss,
                                    const int32_t* __restrict__ row_len, const int32_t* __restrict__ acc_nodes,
                                    const int32_t* __restrict__ acc_len, int32_t dcap) {
    __shared__ int32_t path[FG_MAX_PATH];
    const int32_t b = blockIdx.x;
    const int32_t a = min(acc_len[b], FG_MAX_PATH);
    if (threadIdx.x < FG_MAX_PATH) path[threadIdx.x] = threadIdx.x < a ? acc_nodes[(int64_t)b * dcap + threadIdx.x] : 0;
    __syncthreads();
    if (a <= 0) return;
    compact_row(kv, n_layers, elem_bytes, n_heads, head_dim, sb, sh, ss, b, row_len[b], path, a);
}

using AcceptKernel = void (*)(AcceptParams, KvPtrs);

static cudaError_t launch_accept(AcceptKernel kernel, int32_t B, cudaStream_t st, const AcceptParams& p,
                                 const KvPtrs& kv) {
    kernel<<<B, FG_SAMPLE_LANES, 0, st>>>(p, kv);
    return cudaSuccess;
}

static cudaError_t launch_accept_cluster(AcceptKernel kernel, int32_t B, cudaStream_t st, const AcceptParams& p,
                                         const KvPtrs& kv) {
    const int64_t ebuf = cluster_ebuf_bytes(p.vocab);
    if (ebuf > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ebuf);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)B * kAcceptCtas);
    cfg.blockDim = dim3(kAcceptClusterThreads);
    cfg.dynamicSmemBytes = (size_t)ebuf;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kAcceptCtas;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, p, kv);
}

static bool kv_aligned(int32_t elem_bytes, int32_t head_dim, int64_t sb, int64_t sh, int64_t ss) {
    const int64_t eb = elem_bytes;
    return (head_dim * eb) % 16 == 0 && (sb * eb) % 16 == 0 && (sh * eb) % 16 == 0 && (ss * eb) % 16 == 0;
}

}  // namespace fg

using namespace fg;

extern "C" fg_status fg_accept_extract(const fg_accept_args* a, void* stream) {
    if (!a) return FG_EINVAL;
    if (a->B == 0) return FG_OK;
    if (a->B < 0 || !a->logits || !a->slot || !a->tokens || !a->parents || !a->uniforms || !a->row_len ||
        !a->acc_tokens || !a->acc_nodes || !a->acc_len || !a->correction || !a->pending || !a->last_node ||
        !a->finished || a->vocab <= 0 || a->nmax <= 0)
        return FG_EINVAL;
    if (a->dcap <= 0 || a->dcap > FG_MAX_PATH || a->nmax > 4096 || a->n_layers > FG_MAX_LAYERS) return FG_ECAPACITY;
    if (a->n_layers > 0) {
        if (!a->k_layers || !a->v_layers || (a->kv_elem_bytes != 2 && a->kv_elem_bytes != 4)) return FG_EINVAL;
        if (!kv_aligned(a->kv_elem_bytes, a->head_dim, a->kv_stride_b, a->kv_stride_h, a->kv_stride_s))
            return FG_EINVAL;
    }
    if (a->hidden_out && (!a->tree_hidden || ((int64_t)a->hidden_dim * a->hidden_elem_bytes) % 16 != 0))
        return FG_EINVAL;
    if (a->kv_rows && a->kv_batch <= 0) return FG_EINVAL;
    AcceptParams p;
    p.logits = a->logits;
    p.logits_row_stride = a->logits_row_stride;
    p.vocab = a->vocab;
    p.slot = a->slot;
    p.tokens = a->tokens;
    p.parents = a->parents;
    p.parent_stride = a->parent_stride;
    p.n_nodes = a->n_nodes;
    p.n_nodes_shared = a->n_nodes_shared;
    p.nmax = a->nmax;
    p.uniforms = a->uniforms;
    p.u_stride = a->u_stride;
    p.do_sample = a->do_sample;
    p.temperature = a->temperature;
    p.top_p = a->top_p;
    p.top_k = a->top_k;
    p.eos_id = a->eos_id;
    p.max_length = a->max_length;
    p.row_len = a->row_len;
    p.update_len = a->update_len;
    p.active = a->active;
    p.dcap = a->dcap;
    p.acc_tokens = a->acc_tokens;
    p.acc_nodes = a->acc_nodes;
    p.acc_len = a->acc_len;
    p.correction = a->correction;
    p.pending = a->pending;
    p.last_node = a->last_node;
    p.finished = a->finished;
    p.n_layers = a->n_layers;
    p.kv_elem_bytes = a->kv_elem_bytes;
    p.n_kv_heads = a->n_kv_heads;
    p.head_dim = a->head_dim;
    p.kv_stride_b = a->kv_stride_b;
    p.kv_stride_h = a->kv_stride_h;
    p.kv_stride_s = a->kv_stride_s;
    p.tree_hidden = a->tree_hidden;
    p.hidden_out = a->hidden_out;
    p.hidden_dim = a->hidden_dim;
    p.hidden_elem_bytes = a->hidden_elem_bytes;
    p.kv_rows = a->kv_rows;
    p.kv_batch = a->kv_batch;
    p.drawn = nullptr;
    p.acc_total = a->acc_total;
    p.round_counter = a->round_counter;
    const bool parallel = a->drawn != nullptr;
    if (parallel && (!a->internal || !a->depths || a->internal_rows <= 0 || a->parent_stride != 0)) return FG_EINVAL;
    KvPtrs kv;
    for (int l = 0; l < FG_MAX_LAYERS; ++l) {
        kv.k[l] = l < a->n_layers ? a->k_layers[l] : 0;
        kv.v[l] = l < a->n_layers ? a->v_layers[l] : 0;
    }
    cudaStream_t st = (cudaStream_t)stream;
    if (parallel) {
        const int32_t n_static = a->internal_rows / a->B;
        switch (a->logits_dtype) {
            case FG_DTYPE_F32:
                draw_internal_kernel<float><<<a->internal_rows, FG_SAMPLE_LANES, 0, st>>>(
                    p, a->B, a->internal, a->depths, a->plan_out, n_static, a->drawn);
                break;
            case FG_DTYPE_BF16:
                draw_internal_kernel<__nv_bfloat16><<<a->internal_rows, FG_SAMPLE_LANES, 0, st>>>(
                    p, a->B, a->internal, a->depths, a->plan_out, n_static, a->drawn);
                break;
            case FG_DTYPE_F16:
                draw_internal_kernel<__half><<<a->internal_rows, FG_SAMPLE_LANES, 0, st>>>(
                    p, a->B, a->internal, a->depths, a->plan_out, n_static, a->drawn);
                break;
            default:
                return FG_EINVAL;
        }
        const int32_t s = launch_status();
        if (s != FG_OK) return s;
        p.drawn = a->drawn;
    }
    // fg-icdf-v1 draws in the walk run on a cluster of kAcceptCtas CTAs per row
    const bool cuts = sample_cuts(a->do_sample, a->temperature, a->top_p, a->top_k, a->vocab);
    // (the e_i buffer of one chunk group within 96 KB: V up to ~95k x 8 entries)
    const bool clustered = !parallel && a->do_sample && a->temperature > 0.0f && !cuts &&
                           sample_chunk_len(a->vocab) <= kFindWarpMax && cluster_ebuf_bytes(a->vocab) <= 96 * 1024;
    cudaError_t e = cudaSuccess;
    switch (a->logits_dtype) {
        case FG_DTYPE_F32:
            e = clustered ? launch_accept_cluster(accept_extract_kernel<float, kAcceptCtas>, a->B, st, p, kv)
                          : launch_accept(accept_extract_kernel<float, 1>, a->B, st, p, kv);
            break;
        case FG_DTYPE_BF16:
            e = clustered ? launch_accept_cluster(accept_extract_kernel<__nv_bfloat16, kAcceptCtas>, a->B, st, p, kv)
                          : launch_accept(accept_extract_kernel<__nv_bfloat16, 1>, a->B, st, p, kv);
            break;
        case FG_DTYPE_F16:
            e = clustered ? launch_accept_cluster(accept_extract_kernel<__half, kAcceptCtas>, a->B, st, p, kv)
                          : launch_accept(accept_extract_kernel<__half, 1>, a->B, st, p, kv);
            break;
        default:
            return FG_EINVAL;
    }
    if (e != cudaSuccess) {
        set_cuda_error(e);
        return FG_ECUDA;
    }
    return launch_status();
}

extern "C" fg_status fg_extract_path(int32_t n_layers, const uint64_t* k_layers, const uint64_t* v_layers,
                                     int32_t kv_elem_bytes, int32_t B, int32_t n_kv_heads, int32_t head_dim,
                                     int64_t stride_b, int64_t stride_h, int64_t stride_s, const int32_t* row_len,
                                     const int32_t* acc_nodes, const int32_t* acc_len, int32_t dcap, void* stream) {
    if (B == 0 || n_layers == 0) return FG_OK;
    if (B < 0 || !k_layers || !v_layers || !row_len || !acc_nodes || !acc_len) return FG_EINVAL;
    if (n_layers > FG_MAX_LAYERS || dcap <= 0 || dcap > FG_MAX_PATH) return FG_ECAPACITY;
    if ((kv_elem_bytes != 2 && kv_elem_bytes != 4) || !kv_aligned(kv_elem_bytes, head_dim, stride_b, stride_h, stride_s))
        return FG_EINVAL;
    KvPtrs kv;
    for (int l = 0; l < FG_MAX_LAYERS; ++l) {
        kv.k[l] = l < n_layers ? k_layers[l] : 0;
        kv.v[l] = l < n_layers ? v_layers[l] : 0;
    }
    extract_path_kernel<<<B, 256, 0, (cudaStream_t)stream>>>(kv, n_layers, kv_elem_bytes, n_kv_heads, head_dim,
                                                             stride_b, stride_h, stride_s, row_len, acc_nodes,
                                                             acc_len, dcap);
    return launch_status();
}

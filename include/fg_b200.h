/*
 * fg_b200.h -- C ABI of the B200 (sm_100a) MEDUSA tree-verify hot path.
 *
 * One MEDUSA tree-verify iteration of FlashGRPO's speculative rollout step:
 * proposal candidates -> dense candidate tree -> tree attention inside the
 * verify forward -> exact_target acceptance + extract_path KV compaction.
 * Reference: ihbkaiser/ss-GRPO, package flashgrpo_b200 (paths below are
 * inside that project).  The reference has no C/FFI layer; each entry point
 * replaces the Python/PyTorch call named in its comment, and the Python
 * package in ss-grpo_b200/flashgrpo_b200 binds them with ctypes.
 *
 * Conventions
 *   - Every entry point returns an fg_status (0 = FG_OK) and never syncs the
 *     host; work is enqueued on `stream` (a cudaStream_t passed as void*).
 *   - No entry point allocates device memory.  Callers own every buffer;
 *     scratch is passed as `workspace` with a matching *_workspace_size().
 *   - Pointers are device pointers unless the comment says "host".
 *   - Tensors are row-major; strides are in elements.
 *   - Kernels that wait on shared-memory barriers give up after about one
 *     second, record FG_ETIMEOUT in the device error word (fg_read_device_error)
 *     and return instead of hanging.
 *
 * Sampler specification "fg-icdf-v1" (shared by the kernels and the CPU
 * checker; the reference samples with torch.multinomial,
 * flashgrpo_b200/decoding/acceptance.py:56-60, so supplied uniforms need a
 * written definition to be reproducible):
 *   u      = (Philox4x32-10(counter = (seq_id, round, draw, 0),
 *                           key = (seed lo32, seed hi32)).x >> 8) * 2^-24
 *   x_i    = float(logit_i) / T            (IEEE division, only when T > 0)
 *   m      = max_i x_i;  e_i = fg_exp(x_i - m)   (Cody-Waite + degree-7
 *            Taylor with fused Horner steps; 0 below -86)
 *   the vocabulary is cut into 512 contiguous chunks of
 *   C = roundup8(ceil(V / 512)) entries; c_i = left-to-right fp32 prefix sum
 *   of e inside the chunk of i; s_t = chunk total;
 *   P_0 = 0, P_{t+1} = P_t + s_t (sequential), target = u * P_512;
 *   t* = the chunk with P_t <= target < P_{t+1};
 *   token = first i of chunk t* with P_t* + c_i > target.
 *   Greedy (do_sample == 0 or T == 0): first index of the maximum logit.
 * Nucleus variant "fg-icdf-v1n" (0 < top_p < 1), on exact integer masses:
 *   q_i = trunc(e_i * 2^40) (uint64), Z = sum q_i,
 *   P = trunc(double(top_p) * double(Z)); order entries by key descending,
 *   index ascending, key = order-preserving image of x (-0 as +0); the
 *   boundary K* is the first position whose cumulative mass exceeds P (mass
 *   S there); kept = entries before or at K*;
 *   t = trunc(double(u) * double(S)); token = first index (ascending) among
 *   kept entries whose running kept mass exceeds t.
 * Top-k variant "fg-icdf-v1k" (0 < top_k < V; the top_k branch of
 * sample_from_logits, acceptance.py:68-79): the K-set is the first top_k
 *   entries of that order, Zk its mass; with 0 < top_p < 1,
 *   P = trunc(double(top_p) * double(Zk)) and K*, S as above, otherwise K* is
 *   the K-set's last entry and S = Zk; kept, t and token as above.  Equal
 *   logits are ordered by index (torch.topk leaves their order unspecified).
 */
#ifndef FG_B200_H_
#define FG_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t fg_status;
#define FG_OK 0
#define FG_EINVAL 1       /* bad argument (shape, dtype, null pointer, alignment) */
#define FG_ECAPACITY 2    /* a size exceeds a compile-time or buffer capacity */
#define FG_ETIMEOUT 3     /* a device-side wait gave up */
#define FG_ECUDA 4        /* a CUDA launch/runtime call failed; see fg_last_cuda_error */
#define FG_EUNSUPPORTED 5 /* configuration not implemented (e.g. a dtype a kernel does not take) */

#define FG_DTYPE_F32 0
#define FG_DTYPE_BF16 1
#define FG_DTYPE_F16 2

#define FG_MAX_TREE_NODES 128 /* nodes per candidate tree (ancestor mask words = 4) */
#define FG_MAX_DEPTHS 8       /* MEDUSA heads / tree depth below the root */
#define FG_MAX_TOPK 16        /* candidates per head and row */
#define FG_MAX_PATH 16        /* accepted tokens per row and round */
#define FG_MAX_LAYERS 128     /* layers addressed by one compaction call */

/* ------------------------------------------------------------ housekeeping */
const char *fg_version(void);
const char *fg_status_string(fg_status status);
/* Last cudaError_t recorded by any entry point in this process. */
int32_t fg_last_cuda_error(void);
/* Synchronously reads (and with clear != 0 resets) the device error word of
 * the current device: 0 or the first FG_* status a kernel recorded. */
fg_status fg_read_device_error(int32_t *host_out, int32_t clear);
/* Failure-path check: a kernel waits on *flag (device int32) becoming
 * nonzero for at most timeout_ns, then writes FG_OK or FG_ETIMEOUT to
 * *status_out (device int32).  Used to test bounded device waits. */
fg_status fg_wait_flag(const int32_t *flag, int64_t timeout_ns, int32_t *status_out, void *stream);

/* ------------------------------------------------------------- sampling */
/* out[r * n_draws + d] = u(seed, seq_ids[r], round, d) with
 * round = round_idx + (round_dev ? *round_dev : 0); round_dev (nullable,
 * device int32) lets a captured CUDA graph advance the round on the device.
 * Draw 0 is the root sample of a round, draw 1 + s is acceptance step s. */
fg_status fg_philox_uniforms(uint64_t seed, const int32_t *seq_ids, int32_t n_rows, int32_t round_idx,
                             const int32_t *round_dev, int32_t n_draws, float *out, void *stream);

/* One token per row of logits [n_rows, row_stride] (dtype FG_DTYPE_*),
 * uniform uniforms[r * u_stride]: fg-icdf-v1 for top_p >= 1 (or <= 0) and
 * top_k outside (0, vocab), the nucleus variant fg-icdf-v1n for
 * 0 < top_p < 1 (the kept set of logits_to_probs, acceptance.py:7-31, on
 * exact integer masses), the top-k variant fg-icdf-v1k for 0 < top_k < vocab
 * (with or without a top_p cut).  forced (nullable): rows with forced[r] >= 0
 * take that token instead (pending correction tokens).  Replaces
 * sample_from_logits (flashgrpo_b200/decoding/acceptance.py:34-130) for the
 * root token of a round (flashgrpo_b200/decoding/flash_medusa_decoder.py:1717-1743). */
fg_status fg_sample_rows(const void *logits, int32_t dtype, int64_t row_stride, int32_t vocab, int32_t n_rows,
                         const float *uniforms, int64_t u_stride, int32_t do_sample, float temperature,
                         float top_p, int32_t top_k, const int32_t *forced, int32_t *out_tokens, void *stream);

/* Per row: the k best entries ordered by (value descending, index
 * ascending), the row maximum and logsumexp (rounded to the logits dtype,
 * as torch.logsumexp returns it; out_lse may be NULL to skip it, as only
 * adaptive trees use it).  k <= FG_MAX_TOPK.  Without out_lse every row
 * runs on a cluster of 8 CTAs (a threshold selection over vocabulary
 * slices); the result is the same.  Replaces torch.topk in
 * build_batch_trees (flashgrpo_b200/decoding/medusa_tree.py:767) and the
 * confidence reductions (flash_medusa_decoder.py:1034-1040). */
fg_status fg_row_topk(const void *logits, int32_t dtype, int64_t row_stride, int32_t vocab, int32_t n_rows,
                      int32_t k, int32_t *out_idx, float *out_val, float *out_max, float *out_lse, void *stream);

/* The tied lm_head of the proposal rows on the tensor cores with the top-k
 * fused: logits[r, v] = bf16(x[r, :] . w[v, :]) for x [M, H] (M <= 256,
 * H a multiple of 64), w [V, H] (bf16, row strides x_ld / w_ld elements).
 * Rows [0, n_logit_rows) write their logits to `logits` (row stride
 * logits_ld); rows [topk_row0, M) produce, in row order from topk_row0, what
 * fg_row_topk returns on those logits (k best by value desc / index asc,
 * maximum, logsumexp rounded to bf16 when out_lse != NULL) without writing
 * them.  topk_row0 == M skips the top-k.  workspace:
 * fg_lm_head_topk_workspace_size bytes (no zero-fill needed).  Replaces the
 * concat-heads lm_head of _medusa_logits_for_last_hidden
 * (flashgrpo_b200/decoding/flash_medusa_decoder.py:906-1005) followed by the
 * torch.topk of build_batch_trees (medusa_tree.py:767) and the confidence
 * reductions (flash_medusa_decoder.py:1034-1040).  dtype FG_DTYPE_BF16 only. */
size_t fg_lm_head_topk_workspace_size(int32_t M, int32_t V, int32_t topk_row0, int32_t k);
fg_status fg_lm_head_topk(const void *x, int32_t dtype, int64_t x_ld, int32_t M, int32_t H, const void *w,
                          int64_t w_ld, int32_t V, int32_t n_logit_rows, void *logits, int64_t logits_ld,
                          int32_t topk_row0, int32_t k, int32_t *out_idx, float *out_val, float *out_max,
                          float *out_lse, void *workspace, size_t workspace_bytes, void *stream);

/* One MEDUSA head (heads.{i}.norm and heads.{i}.fc of a medusa_heads.pt
 * state dict): device pointers to the LayerNorm weight and bias [H] and the
 * fc weight [H, H] (nn.Linear layout, out x in, row-major) and bias [H]. */
typedef struct fg_medusa_head {
    const void *norm_w;
    const void *norm_b;
    const void *fc_w;
    const void *fc_b;
} fg_medusa_head;

/* The whole MEDUSA proposal step of a round on the tensor cores.
 * x is [(1 + n_heads) * B, H] bf16, row-major: rows [0, B) hold the root
 * hidden states on entry; rows [(i + 1) B, (i + 2) B) receive head i's
 * projected states h + silu(fc(layer_norm(h)))
 * (MedusaPredictionHead.project_hidden, flashgrpo_b200/models/
 * medusa_heads.py:240-244; the fc runs as a split-K tcgen05 GEMM whose
 * fp32 partial sums are combined with the bias, SiLU and residual in one
 * pass).  Then the tied lm_head over all (1 + n_heads) B rows
 * (fg_lm_head_topk): the root rows' logits go to root_logits (row stride
 * logits_ld; NULL skips them) and every head row keeps its k best tokens,
 * maximum and (out_lse != NULL) logsumexp in out_* rows i * B + b.
 * Replaces _medusa_logits_for_last_hidden
 * (flashgrpo_b200/decoding/flash_medusa_decoder.py:906-1005) with the
 * torch.topk of build_batch_trees (medusa_tree.py:767) and the confidence
 * reductions (flash_medusa_decoder.py:1034-1040).  heads: host array of
 * n_heads entries (n_heads >= 0; 0 computes the root logits only).
 * (1 + n_heads) B <= 256, H a multiple of 64 and at most 8192, dtype
 * FG_DTYPE_BF16 only, head weights 16-byte aligned (fc_b 8-byte);
 * workspace: fg_medusa_propose_workspace_size bytes, 256-byte aligned. */
size_t fg_medusa_propose_workspace_size(int32_t B, int32_t H, int32_t V, int32_t n_heads, int32_t k);
fg_status fg_medusa_propose(void *x, int32_t dtype, int32_t B, int32_t H, const fg_medusa_head *heads,
                            int32_t n_heads, float eps, const void *lm_head_w, int64_t w_ld, int32_t V,
                            void *root_logits, int64_t logits_ld, int32_t k, int32_t *out_idx, float *out_val,
                            float *out_max, float *out_lse, void *workspace, size_t workspace_bytes, void *stream);

/* The ChainDraftCell of a Chain-MEDUSA checkpoint (chain_cell.* entries):
 * device pointers, bf16.  norms [H]; state_proj / token_proj [bottleneck, H]
 * and out_proj [H, bottleneck] in nn.Linear layout (out x in, row-major);
 * out_b [H]; gate: one element. */
typedef struct fg_chain_cell {
    const void *state_norm_w;
    const void *state_norm_b;
    const void *token_norm_w;
    const void *token_norm_b;
    const void *state_proj_w;
    const void *token_proj_w;
    const void *out_proj_w;
    const void *out_proj_b;
    const void *gate;
    int32_t bottleneck;
} fg_chain_cell;

/* One level of a chain proposal on the tensor cores.  Rows are grouped by
 * sequence: row r = b * n_child + j (b < n_seq, j < n_child) extends parent
 * state s = state[b * n_parent + j / fanout] with token
 * t = tokens[b * tok_ld + j] (t in [0, V): the embedding table has the
 * lm_head's V rows; others record FG_EINVAL in the device error word and
 * read row 0):
 *   state_out[r] = s + sigmoid(gate) * out_proj(silu(state_proj(LN_s(s)) + token_proj(LN_t(embed[t]))))
 * (ChainDraftCell.forward, flashgrpo_b200/models/medusa_heads.py:154-160,
 * rounded to bf16 after every op as the reference's bf16 module does; the
 * three projections run as split-K tcgen05 GEMMs), then, when k > 0, what
 * fg_lm_head_topk returns for every state_out row (k best, maximum,
 * logsumexp when out_lse != NULL) -- the per-parent candidates of the next
 * level.  Replaces one iteration of the chain loop of
 * _build_chain_batch_trees (flashgrpo_b200/decoding/flash_medusa_decoder.py:
 * 1141-1261).  state [n_seq * n_parent, H], state_out [n_seq * n_child, H]
 * and embed rows (stride embed_ld) are bf16 with contiguous rows; state_out
 * must not overlap state.  n_child <= n_parent * fanout <= tok_ld * fanout;
 * any number of rows (processed 256 at a time); H and bottleneck multiples
 * of 64, H at most 8192; dtype FG_DTYPE_BF16 only; workspace:
 * fg_chain_step_workspace_size bytes for M = n_seq * n_child rows, 256-byte
 * aligned. */
size_t fg_chain_step_workspace_size(int32_t M, int32_t H, int32_t bottleneck, int32_t V, int32_t k);
fg_status fg_chain_step(const void *state, const int32_t *tokens, int32_t tok_ld, int32_t n_seq, int32_t n_parent,
                        int32_t fanout, int32_t n_child, const void *embed, int64_t embed_ld, int32_t H,
                        int32_t dtype, const fg_chain_cell *cell, float eps, void *state_out, const void *lm_head_w,
                        int64_t w_ld, int32_t V, int32_t k, int32_t *out_idx, float *out_val, float *out_max,
                        float *out_lse, void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------ tree build */
typedef struct fg_plan_params {
    int32_t tree_mode;          /* 0 = "fixed", 1 = "concurrency_aware", 2 = explicit
                                   (fixed_topk and max_tree_nodes_per_seq taken as a
                                   finished TreePlan: no trimming, no planning) */
    int32_t active_batch_size;  /* rows in the round (plan_tree active_batch_size) */
    int32_t num_medusa_heads;
    int32_t cpeak_nodes;
    int32_t min_tree_nodes_per_seq;
    int32_t max_tree_nodes_per_seq;
    int32_t max_tree_depth;
    int32_t n_fixed;            /* entries of fixed_tree_topk_by_depth */
    int32_t fixed_topk[FG_MAX_DEPTHS];
    int32_t adaptive;           /* adaptive_tree_enabled */
    int32_t n_min;              /* entries of adaptive_min_topk_by_depth */
    int32_t adaptive_min_topk[FG_MAX_DEPTHS];
    int32_t confidence_metric;  /* 0 = "top1_prob", 1 = "margin" */
    float confidence_quantile;
    double confidence_low;
    double confidence_high;
    double depth_weight[FG_MAX_DEPTHS]; /* host: max(decay, 1e-3) ** d */
    double log_gain[65];        /* host: log1p(v) - log(v) for v = 0..64 (index 0 unused) */
} fg_plan_params;

/* Plans and builds the shared-topology dense MEDUSA tree of one round:
 * plan_tree (flashgrpo_b200/decoding/medusa_tree.py:342-459, dense layout),
 * optional adaptive top-k (flash_medusa_decoder.py:1021-1095, from head_max /
 * head_lse / cand_val), the BFS expansion with budget truncation
 * (medusa_tree.py:758-799), the ancestor-only mask of
 * build_tree_attention_inputs (flashgrpo_b200/decoding/tree_attention.py:6-67)
 * as bits, logical positions row_len + depth - 1 (:58) and the packed
 * internal-node logits layout (flash_medusa_decoder.py:1097-1118).
 *   root [B], cand_idx/cand_val [n_heads][B][kmax] (fg_row_topk output),
 *   head_max/head_lse [n_heads][B] (adaptive only), row_len [B].
 * Outputs: tokens [B][nmax], positions [B][nmax], slot [B][nmax]
 * (b * n_internal + rank, or -1 for leaves), parents/depths [nmax],
 * anc_bits [nmax][4] (bit j of node i: j is i or an ancestor of i),
 * internal [nmax] (node ids with children), plan_out [16] =
 * {budget, n_depth, topk[8], n_nodes, n_internal, 0...}.
 * Rows share one topology; nmax <= FG_MAX_TREE_NODES. */
fg_status fg_build_tree(const fg_plan_params *plan, const int32_t *root, const int32_t *cand_idx,
                        const float *cand_val, const float *head_max, const float *head_lse, int32_t n_heads,
                        int32_t kmax, int32_t B, int32_t nmax, int32_t logits_dtype, const int32_t *row_len,
                        int32_t *tokens, int32_t *positions, int32_t *slot, int32_t *parents, int32_t *depths,
                        uint32_t *anc_bits, int32_t *internal, int32_t *plan_out, void *stream);

/* -------------------------------------------------------- tree attention */
typedef struct fg_kv_layer {
    void *k;          /* [batch, Hkv, capacity, D] addressed with the strides below */
    void *v;
    int64_t stride_b; /* elements */
    int64_t stride_h;
    int64_t stride_s;
    int32_t capacity; /* positions per (row, head) */
    /* Row map for rounds over a subset of the cache's rows (finished rows
     * retired without moving any K/V): call row b uses cache row rows[b].
     * NULL = identity (then batch is ignored and the cache has the call's B
     * rows).  A mapped row outside [0, batch) is skipped and records
     * FG_EINVAL in the device error word. */
    const int32_t *rows;
    int32_t batch;    /* rows of the cache when rows != NULL */
} fg_kv_layer;

/* Flash-decoding GQA attention of the tree queries of one layer:
 *   q   [B, n_nodes, Hq, D]  (RoPE applied), out [B, n_nodes, Hq, D]
 *   key/value of row b: prefix slots [0, kv_len[b]) plus the tree nodes at
 *   slots kv_len[b] + j; node i attends to every prefix slot and to tree
 *   slot j iff bit j of anc_bits[i] is set (the additive mask of
 *   tree_attention.py:6-67 as bits).
 * Replaces HF eager/SDPA attention with the dense 4D mask inside
 * forward_tree (flashgrpo_b200/models/qwen_flashgrpo_wrapper.py:220-239).
 * dtype FG_DTYPE_BF16 (tensor cores, D = 128, scale > 0) or FG_DTYPE_F32
 * (D <= 128).  The bf16 path reads whole 128-slot tiles: slots from
 * kv_len[b] + n_nodes up to the next multiple of 128 (within capacity) are
 * read with weight 0 and must hold finite values (a zero-filled cache does).
 * num_splits 0 = automatic (from max_kv_len, the longest prefix of the
 * batch), at most 128 (FG_EINVAL above).  workspace: fg_tree_attention_workspace_size bytes for the same
 * arguments (0 when one split suffices), zero-filled before first use (the
 * kernels leave it reusable). */
size_t fg_tree_attention_workspace_size(int32_t B, int32_t n_nodes, int32_t n_q_heads, int32_t n_kv_heads,
                                        int32_t head_dim, int32_t num_splits, int32_t max_kv_len);
fg_status fg_tree_attention(const void *q, int32_t dtype, const fg_kv_layer *kv, const int32_t *kv_len,
                            const uint32_t *anc_bits, int32_t B, int32_t n_nodes, int32_t n_q_heads,
                            int32_t n_kv_heads, int32_t head_dim, float scale, void *out, void *workspace,
                            size_t workspace_bytes, int32_t num_splits, int32_t max_kv_len, void *stream);

/* Same attention, for callers that cannot allocate device memory: a caller
 * binding this ABI from another language without a device allocator, or
 * living under a memory manager that owns the GPU, where cudaMalloc would
 * fail or synchronize the device mid-round.  No counterpart in the
 * reference.  The split-K scratch comes from one fixed array inside the
 * library (FG_NOALLOC_SCRATCH_BYTES, held by every GPU that loads the
 * library until exit); needs beyond it return FG_ECAPACITY.  The first call
 * on a device looks the array up (make it before any stream capture; after a
 * cudaDeviceReset of that device the looked-up address is stale); calls
 * share the array, so calls that overlap on the GPU race.  A bf16 call that
 * splits the KV range clears the split counters with a memset on the stream
 * first, so it does not overlap the preceding kernel the way
 * fg_tree_attention does; fp32 calls need no scratch.  Allocates nothing. */
#define FG_NOALLOC_SCRATCH_BYTES (32u << 20)
fg_status fg_tree_attention_noalloc(const void *q, int32_t dtype, const fg_kv_layer *kv, const int32_t *kv_len,
                                    const uint32_t *anc_bits, int32_t B, int32_t n_nodes, int32_t n_q_heads,
                                    int32_t n_kv_heads, int32_t head_dim, float scale, void *out,
                                    int32_t num_splits, int32_t max_kv_len, void *stream);

/* ------------------------------------------------ acceptance + extraction */
typedef struct fg_accept_args {
    const void *logits;        /* tree logits rows (packed internal nodes) */
    int32_t logits_dtype;
    int64_t logits_row_stride;
    int32_t vocab;
    const int32_t *slot;       /* [B][nmax]: node -> logits row, -1 = none */
    const int32_t *tokens;     /* [B][nmax] */
    const int32_t *parents;    /* [B][parent_stride]; parent_stride 0 = shared */
    int32_t parent_stride;
    const int32_t *n_nodes;    /* [B] or NULL (then n_nodes_shared) */
    int32_t n_nodes_shared;
    int32_t nmax;
    const float *uniforms;     /* walk step s of row b uses uniforms[b * u_stride + s] */
    int32_t u_stride;
    int32_t B;
    int32_t do_sample;
    float temperature;
    float top_p;               /* 0 < top_p < 1: nucleus draws (fg-icdf-v1n) */
    int32_t top_k;             /* 0 < top_k < vocab: top-k draws (fg-icdf-v1k); 0: no cut */
    int32_t eos_id;
    int32_t max_length;
    int32_t *row_len;          /* [B] logical length before the round; advanced if update_len */
    int32_t update_len;
    int32_t *active;           /* [B] or NULL; rows with 0 accept nothing; a row
                                  that finishes this round is set to 0 */
    int32_t dcap;              /* columns of acc_tokens / acc_nodes, <= FG_MAX_PATH */
    int32_t *acc_tokens;       /* [B][dcap], -1 padded */
    int32_t *acc_nodes;        /* [B][dcap], -1 padded */
    int32_t *acc_len;          /* [B] */
    int32_t *correction;       /* [B] target sample that missed, -1 none */
    int32_t *pending;          /* [B] next round's forced root, -1 none */
    int32_t *last_node;        /* [B] */
    int32_t *finished;         /* [B] */
    /* KV compaction (n_layers = 0 skips it) */
    int32_t n_layers;
    const uint64_t *k_layers;  /* host array [n_layers] of device pointers */
    const uint64_t *v_layers;
    int32_t kv_elem_bytes;     /* 2 or 4 */
    int32_t n_kv_heads;
    int32_t head_dim;
    int64_t kv_stride_b;
    int64_t kv_stride_h;
    int64_t kv_stride_s;
    /* next-round hidden state gather (hidden_out = NULL skips it) */
    const void *tree_hidden;   /* [B][nmax][hidden_dim] */
    void *hidden_out;          /* [B][hidden_dim] */
    int32_t hidden_dim;
    int32_t hidden_elem_bytes;
    /* compaction row map (see fg_kv_layer.rows): row b compacts cache row
     * kv_rows[b] of kv_batch rows; NULL = identity */
    const int32_t *kv_rows;
    int32_t kv_batch;
    /* Parallel draws (drawn != NULL; shared topology only): before the walk,
     * one CTA per packed logits row j < internal_rows draws the target token
     * at internal node internal[j % n_int] of row j / n_int with uniform
     * u[b][depths[node] - 1] -- the draw the walk would make there -- into
     * drawn[j]; the walk then reads them.  n_int = plan_out[11] (fg_build_tree's
     * plan) when plan_out != NULL, else internal_rows / B.  Same tokens as the
     * sequential walk, with every internal node's draw done at once. */
    const int32_t *internal;   /* [nmax] node ids with children (fg_build_tree) */
    const int32_t *depths;     /* [nmax] */
    const int32_t *plan_out;   /* [16] or NULL */
    int32_t internal_rows;     /* packed logits rows = grid of the draws */
    int32_t *drawn;            /* [internal_rows] int32 scratch, or NULL */
    /* Round counters, each NULL to skip it: *acc_total += the rows' acc_len
     * (the round's accepted tokens), *round_counter += 1 (the round index the
     * next fg_philox_uniforms call reads). */
    int64_t *acc_total;
    int32_t *round_counter;
} fg_accept_args;

/* One CTA per row (fg-icdf-v1 draws: a cluster of 8 CTAs per row that
 * shares each draw's exponentials, see fg_accept.cu): the exact_target walk
 * of exact_accept_paths_batch
 * (flashgrpo_b200/decoding/acceptance.py:183-267), the post-accept clip /
 * EOS / pending-correction rules (flash_medusa_decoder.py:2289-2343), the
 * extract_path compaction of the accepted slots in every layer
 * (flashgrpo_b200/decoding/kv_extraction.py:34-218, on per-row lengths), and
 * current_hidden = tree_hidden[row, last node] (flash_medusa_decoder.py:2829-2835).
 * With args->drawn set, a first kernel makes every internal node's draw in
 * parallel (see fg_accept_args) and the walk reads them. */
fg_status fg_accept_extract(const fg_accept_args *args, void *stream);

/* Compaction alone, for callers that keep their own tree walk:
 * moves slots row_len[b] + acc_nodes[b][j] to row_len[b] + j, j < acc_len[b],
 * in every layer (extract_accepted_path_kv, kv_extraction.py:87-218). */
fg_status fg_extract_path(int32_t n_layers, const uint64_t *k_layers, const uint64_t *v_layers,
                          int32_t kv_elem_bytes, int32_t B, int32_t n_kv_heads, int32_t head_dim, int64_t stride_b,
                          int64_t stride_h, int64_t stride_s, const int32_t *row_len, const int32_t *acc_nodes,
                          const int32_t *acc_len, int32_t dcap, void *stream);

/* ------------------------------------------------- verify-forward helpers */
/* RoPE at the tree positions and the tree K/V write at the cache tail:
 *   qkv [B * n_nodes, (Hq + 2 Hkv) * D] (projection output, bias added),
 *   positions [B][n_nodes], inv_freq [D / 2] (fp32), q_out [B, n_nodes, Hq, D],
 *   K/V of node j of row b go to slot kv_len[b] + j of `kv`.
 * Replaces apply_rotary_pos_emb + DynamicCache.update (torch.cat) inside
 * the verify forward (transformers Qwen2/Llama attention, called from
 * qwen_flashgrpo_wrapper.py:150-186).  dtype bf16/f16 rounds like the
 * reference's half-precision arithmetic; f32 stays in f32. */
/* cos_sin (nullable): the table fg_rope_table made for these positions; the
 * kernel then reads it instead of evaluating cos/sin (same values). */
fg_status fg_rope_kv_write(const void *qkv, int32_t dtype, const int32_t *positions, const float *inv_freq,
                           float attention_scaling, int32_t B, int32_t n_nodes, int32_t n_q_heads,
                           int32_t n_kv_heads, int32_t head_dim, const int32_t *kv_len, const fg_kv_layer *kv,
                           void *q_out, const void *cos_sin, void *stream);
/* cos(pos * inv_freq) * attention_scaling and the sine, rounded to `dtype`
 * like the reference's rotary embedding, for every (token, frequency):
 * cos_sin [2][n_tokens][half] (cosines, then sines).  Positions do not change
 * between the layers of a round, so one table serves them all. */
fg_status fg_rope_table(const int32_t *positions, int32_t n_tokens, const float *inv_freq, int32_t half,
                        float attention_scaling, int32_t dtype, void *cos_sin, void *stream);
/* y = weight * (x * rsqrt(mean(x^2) + eps)) per row (Qwen2RMSNorm / LlamaRMSNorm). */
fg_status fg_rmsnorm(const void *x, const void *weight, int32_t dtype, int32_t n_rows, int32_t dim, float eps,
                     void *y, void *stream);
/* y = layer_norm(x) * weight + bias per row (MEDUSA head norm, eps 1e-5). */
fg_status fg_layernorm(const void *x, const void *weight, const void *bias, int32_t dtype, int32_t n_rows,
                       int32_t dim, float eps, void *y, void *stream);
/* act[t, j] = bf16(bf16(silu(bf16(g))) * bf16(u)) with g = x[t] . w[j] and
 * u = x[t] . w[I + j]: the MLP's act_fn(gate_proj(x)) * up_proj(x) on the
 * tensor cores with SiLU-gating in the GEMM epilogue, so the [T, 2I]
 * gate/up tensor of fg_silu_mul is never written.  x [T, H] and w_gate_up
 * [2I, H] (gate_proj rows, then up_proj rows) bf16 with contiguous rows, act
 * [T, I]; H a multiple of 64, I a multiple of 16; dtype FG_DTYPE_BF16 only.
 * Replaces the gate/up GEMM and act_fn of the HF Qwen2/Llama MLP inside
 * _forward_decoder (flashgrpo_b200/models/qwen_flashgrpo_wrapper.py:150-186). */
fg_status fg_gate_up_silu(const void *x, int32_t dtype, int32_t T, int32_t H, const void *w_gate_up, int32_t I,
                          void *act, void *stream);
/* The verify forward's dense projections on the tensor cores with their
 * consumer fused into the epilogue: D = x w^T for x [M, K] (tokens) and
 * w [N, K] (nn.Linear layout), bf16 with contiguous rows, fp32 accumulation:
 *   FG_EPI_STORE   out = bf16(D + bias)           (bias nullable)
 *   FG_EPI_RESID   out = bf16(resid + D + bias)   (resid may equal out)
 *   FG_EPI_SWIGLU  out = bf16(bf16(silu(bf16(g))) * bf16(u)) with g, u the
 *                  rows j and N + j of w ([2N, K]); no bias
 * out / resid rows are ld_out / ld_resid elements apart (multiples of 8).
 * Replaces the addmm / mm projections of the HF Qwen2 / Llama layers inside
 * _forward_decoder (flashgrpo_b200/models/qwen_flashgrpo_wrapper.py:150-186:
 * q/k/v_proj with bias, o_proj + residual, gate/up + act_fn, down_proj +
 * residual) and the lm_head of the packed internal tree nodes
 * (_project_packed_tree_logits, flashgrpo_b200/decoding/flash_medusa_decoder.py:
 * 1120-1139).  Tiles of bm tokens (128, or 256 as two 128-token MMAs
 * sharing each weight box) x bn outputs (a multiple of 16, at most 256; the
 * epilogue's TMEM reads must fit the tile's accumulator, FG_EINVAL
 * otherwise) with the k range cut into `splits` parts (split-K), through a
 * ring holding `stages` 64-wide k chunks (4, 6 or 8 for bm 128, 6 for bm
 * 256), staged two chunks per slot when K / 64 is even and splits <= K / 128
 * (as many two-chunk slots as shared memory holds, at least two), else one;
 * any of bm / bn / splits / stages <= 0 is chosen from the shape.  splits > 1 writes fp32 partials to workspace
 * (fg_linear_workspace_size bytes for the same bm / bn / splits: splits x M x
 * N floats, 2N for SwiGLU) and a second kernel adds them in k order and
 * applies the epilogue.  K a multiple of 64, N a multiple of 8 (of bn for
 * SwiGLU); dtype FG_DTYPE_BF16 only.  Launched as a programmatic dependent
 * of the preceding kernel: it fetches weights before waiting for it. */
#define FG_EPI_STORE 0
#define FG_EPI_RESID 1
#define FG_EPI_SWIGLU 2
size_t fg_linear_workspace_size(int32_t M, int32_t N, int32_t K, int32_t epilogue, int32_t bm, int32_t bn,
                                int32_t splits);
fg_status fg_linear(const void *x, int32_t dtype, int32_t M, int32_t K, const void *w, int32_t N, const void *bias,
                    const void *resid, int64_t ld_resid, void *out, int64_t ld_out, int32_t epilogue, int32_t bm,
                    int32_t bn, int32_t splits, int32_t stages, void *workspace, size_t workspace_bytes,
                    void *stream);
/* out[r, :I] = silu(gu[r, :I]) * gu[r, I:2I] (SwiGLU of the MLP). */
fg_status fg_silu_mul(const void *gu, int32_t dtype, int32_t n_rows, int32_t inter, void *out, void *stream);
/* out = x + silu(y) (residual of MedusaPredictionHead.project_hidden,
 * flashgrpo_b200/models/medusa_heads.py:240-244). */
fg_status fg_silu_residual(const void *x, const void *y, int32_t dtype, int64_t n, void *out, void *stream);
/* out[r] = src[idx[r]] for rows of `row_bytes` bytes (embedding lookup,
 * internal-node hidden gather).  Rows must be 16-byte multiples. */
fg_status fg_gather_rows(const void *src, int64_t src_row_stride_bytes, const int32_t *idx, int32_t n_rows,
                         int64_t row_bytes, void *out, int64_t out_row_stride_bytes, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* FG_B200_H_ */

// fg_tree.cu -- K2: plan + adaptive top-k + dense MEDUSA tree + ancestor bits.
//
// One CTA builds the round's shared tree topology (the plan does not depend
// on the row) and then fills the per-row token/position/slot tables.
// Reference behaviour: plan_tree (flashgrpo_b200/decoding/medusa_tree.py:342-459,
// dense layout), fit_topk_to_budget (:295-339), the adaptive confidence
// mapping (flashgrpo_b200/decoding/flash_medusa_decoder.py:1021-1095),
// build_batch_trees (medusa_tree.py:758-799), build_tree_attention_inputs
// (flashgrpo_b200/decoding/tree_attention.py:6-67) and the packed internal
// logits layout (flash_medusa_decoder.py:1097-1118).
#include "fg_common.cuh"

namespace fg {

constexpr int kTreeThreads = 512;
constexpr int kSortCap = 1024;  // rows sorted per head for the quantile

__device__ int dense_node_count(const int* topk, int n) {
    int total = 1, width = 1;
    for (int d = 0; d < n; ++d) {
        width *= topk[d];
        total += width;
    }
    return total;
}

// Per-depth branching used when fixed_tree_topk_by_depth is empty.
__device__ __forceinline__ int default_topk(int d) { return d == 0 ? 4 : d == 1 ? 3 : d == 2 ? 2 : 1; }

__device__ __forceinline__ int fixed_or_default(const fg_plan_params& p, int d) {
    return p.n_fixed > 0 ? p.fixed_topk[min(d, p.n_fixed - 1)] : default_topk(d);
}

// plan_tree, dense layout.  Writes budget and the per-depth top-k.
__device__ void device_plan(const fg_plan_params& p, int* budget_out, int* topk, int* n_out) {
    const int bsz = max(1, p.active_batch_size);
    int n = 0, budget;
    if (p.tree_mode == 2) {  // explicit: a TreePlan handed over as-is
        budget = p.max_tree_nodes_per_seq;
        for (int d = 0; d < min(p.n_fixed, FG_MAX_DEPTHS); ++d) {
            if (p.fixed_topk[d] <= 0) break;
            topk[n++] = p.fixed_topk[d];
        }
    } else if (p.tree_mode == 0) {  // fixed
        budget = p.max_tree_nodes_per_seq;
        const int nf = min(p.n_fixed, min(p.num_medusa_heads, FG_MAX_DEPTHS));
        for (int d = 0; d < nf; ++d) topk[n++] = max(1, p.fixed_topk[d]);
        while (n > 0 && dense_node_count(topk, n) > budget) {
            topk[n - 1] -= 1;
            if (topk[n - 1] <= 0) --n;
        }
        const int heads = min(n, max(0, p.max_tree_depth - 1));
        n = heads;
    } else {  // concurrency_aware
        budget = max(p.min_tree_nodes_per_seq, min(p.max_tree_nodes_per_seq, p.cpeak_nodes / bsz));
        const int max_heads = min(min(p.num_medusa_heads, FG_MAX_DEPTHS), max(0, p.max_tree_depth - 1));
        if (p.adaptive) {
            int minimum[FG_MAX_DEPTHS];
            int nm = 0;
            for (int d = 0; d < max_heads; ++d) {
                const int mk = max(1, d < p.n_min ? p.adaptive_min_topk[d] : 1);
                minimum[nm] = mk;
                if (dense_node_count(minimum, nm + 1) > budget) break;
                ++nm;
                topk[n++] = max(mk, fixed_or_default(p, d));
            }
        } else {
            int width = 1, used = 1;
            for (int d = 0; d < max_heads; ++d) {
                const int want = fixed_or_default(p, d);
                const int room = budget - used;
                if (room <= 0) break;
                int k = min(max(1, want), max(1, room / width));
                if (used + width * k > budget) k = room / width;
                if (k <= 0) break;
                topk[n++] = k;
                width *= k;
                used += width;
            }
        }
    }
    *budget_out = budget;
    *n_out = n;
}

// _topk_from_confidence: float64 arithmetic in the reference's operation
// order, explicit round-to-nearest so nothing is contracted; Python's round()
// is half-to-even, as rint.
__device__ int topk_from_confidence(const fg_plan_params& p, double conf, int base_k, int depth) {
    base_k = max(1, base_k);
    const int nm = p.n_min > 0 ? p.n_min : 1;
    const int raw_min = p.n_min > 0 ? p.adaptive_min_topk[min(depth, nm - 1)] : 1;
    const int min_k = max(1, min(base_k, raw_min));
    if (base_k <= min_k) return base_k;
    if (!isfinite(conf)) return min_k;
    const double low = p.confidence_low, high = p.confidence_high;
    if (high <= low) return conf >= high ? min_k : base_k;
    if (conf <= low) return base_k;
    if (conf >= high) return min_k;
    const double ratio = __ddiv_rn(__dsub_rn(conf, low), __dsub_rn(high, low));
    const double kf = __dsub_rn((double)base_k, __dmul_rn(ratio, (double)(base_k - min_k)));
    const int k = (int)rint(kf);
    return max(min_k, min(base_k, k));
}

// fit_topk_to_budget with the log-gain and depth-weight tables from the host.
__device__ int fit_topk(const fg_plan_params& p, int* fitted, int n, int budget) {
    budget = max(1, budget);
    int floor_k[FG_MAX_DEPTHS];
    for (int d = 0; d < n; ++d) {
        fitted[d] = max(1, fitted[d]);
        floor_k[d] = max(1, min(fitted[d], d < p.n_min ? p.adaptive_min_topk[d] : 1));
    }
    while (n > 0 && dense_node_count(fitted, n) > budget) {
        int best = -1, best_saved = 0;
        double best_ratio = 0.0;
        const int cur = dense_node_count(fitted, n);
        for (int d = 0; d < n; ++d) {
            const int v = fitted[d];
            if (v <= floor_k[d]) continue;
            fitted[d] = v - 1;
            const int saved = cur - dense_node_count(fitted, n);
            fitted[d] = v;
            const double loss = __dmul_rn(p.depth_weight[d], p.log_gain[min(v, 64)]);
            const double ratio = __ddiv_rn((double)saved, fmax(loss, 1e-9));
            // max over (ratio, saved, depth)
            if (best < 0 || ratio > best_ratio || (ratio == best_ratio && (saved > best_saved ||
                                                                           (saved == best_saved && d > best)))) {
                best = d;
                best_ratio = ratio;
                best_saved = saved;
            }
        }
        if (best >= 0) {
            fitted[best] -= 1;
        } else {
            --n;
        }
    }
    return n;
}

struct TreeSmem {
    int parents[FG_MAX_TREE_NODES];
    int depths[FG_MAX_TREE_NODES];
    int cand[FG_MAX_TREE_NODES];   // candidate rank used by the node
    int rank[FG_MAX_TREE_NODES];   // packed-row rank, -1 for leaves
    uint32_t anc[FG_MAX_TREE_NODES][4];
    int topk[FG_MAX_DEPTHS];
    int n_depth, budget, n_nodes, n_internal;
    float conf[FG_MAX_DEPTHS];
    float sortbuf[kSortCap];
};

__device__ float score_of(const fg_plan_params& p, const float* cand_val, const float* head_max,
                          const float* head_lse, int kmax, int B, int h, int b, int32_t dtype) {
    float s;
    if (p.confidence_metric == 1) {
        const float v0 = cand_val[((int64_t)h * B + b) * kmax + 0];
        const float v1 = kmax > 1 ? cand_val[((int64_t)h * B + b) * kmax + 1] : 0.0f;
        s = kmax > 1 ? __fsub_rn(v0, v1) : v0;
        if (dtype == FG_DTYPE_BF16) s = __bfloat162float(__float2bfloat16_rn(s));
        if (dtype == FG_DTYPE_F16) s = __half2float(__float2half_rn(s));
    } else {
        s = expf(__fsub_rn(head_max[(int64_t)h * B + b], head_lse[(int64_t)h * B + b]));
    }
    if (isnan(s) || isinf(s)) s = 0.0f;
    return s;
}

__global__ void __launch_bounds__(kTreeThreads) build_tree_kernel(
    fg_plan_params p, const int32_t* __restrict__ root, const int32_t* __restrict__ cand_idx,
    const float* __restrict__ cand_val, const float* __restrict__ head_max, const float* __restrict__ head_lse,
    int32_t n_heads, int32_t kmax, int32_t B, int32_t nmax, int32_t dtype, const int32_t* __restrict__ row_len,
    int32_t* __restrict__ tokens, int32_t* __restrict__ positions, int32_t* __restrict__ slot,
    int32_t* __restrict__ parents_out, int32_t* __restrict__ depths_out, uint32_t* __restrict__ anc_out,
    int32_t* __restrict__ internal_out, int32_t* __restrict__ plan_out) {
    __shared__ TreeSmem sm;
    const int tid = threadIdx.x;
    if (tid == 0) {
        int budget, n;
        device_plan(p, &budget, sm.topk, &n);
        sm.budget = budget;
        sm.n_depth = n;
    }
    __syncthreads();
    // ---- adaptive top-k: quantile of per-row confidences, per head
    if (p.adaptive && sm.n_depth > 0 && n_heads > 0) {
        const int hc = min(sm.n_depth, n_heads);
        int pow2 = 1;
        while (pow2 < B) pow2 <<= 1;
        for (int h = 0; h < hc; ++h) {
            for (int i = tid; i < pow2; i += kTreeThreads)
                sm.sortbuf[i] = i < B ? score_of(p, cand_val, head_max, head_lse, kmax, B, h, i, dtype) : INFINITY;
            __syncthreads();
            // bitonic sort ascending
            for (int size = 2; size <= pow2; size <<= 1)
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
                    for (int i = tid; i < pow2; i += kTreeThreads) {
                        const int j = i ^ stride;
                        if (j > i) {
                            const bool up = (i & size) == 0;
                            const float a = sm.sortbuf[i], c = sm.sortbuf[j];
                            if ((a > c) == up) {
                                sm.sortbuf[i] = c;
                                sm.sortbuf[j] = a;
                            }
                        }
                    }
                    __syncthreads();
                }
            if (tid == 0) {
                // torch.quantile, linear: ranks = q * (n - 1) in fp32, lerp between neighbours
                const float q = fminf(1.0f, fmaxf(0.0f, p.confidence_quantile));
                const float ranks = __fmul_rn(q, (float)(B - 1));
                const int below = (int)ranks;
                const int above = (int)ceilf(ranks);
                const float w = __fsub_rn(ranks, (float)below);
                const float lo = sm.sortbuf[below], hi = sm.sortbuf[above];
                const float d = __fsub_rn(hi, lo);
                sm.conf[h] = fabsf(w) < 0.5f ? __fmaf_rn(w, d, lo) : __fmaf_rn(-d, __fsub_rn(1.0f, w), hi);
            }
            __syncthreads();
        }
        if (tid == 0) {
            int adapted[FG_MAX_DEPTHS];
            for (int d = 0; d < hc; ++d) adapted[d] = topk_from_confidence(p, (double)sm.conf[d], sm.topk[d], d);
            const int n = fit_topk(p, adapted, hc, sm.budget);
            for (int d = 0; d < n; ++d) sm.topk[d] = adapted[d];
            sm.n_depth = n;
        }
        __syncthreads();
    }
    // ---- BFS expansion with budget truncation (thread 0; at most 128 nodes)
    if (tid == 0) {
        const int budget = sm.budget;
        const int cap = min(nmax, FG_MAX_TREE_NODES);
        int n = 1;
        sm.parents[0] = -1;
        sm.depths[0] = 1;
        sm.cand[0] = -1;
        int frontier_lo = 0, frontier_hi = 1;  // nodes of the previous depth are contiguous
        int nd = min(sm.n_depth, n_heads);
        bool overflow = false;
        for (int d = 0; d < nd; ++d) {
            const int k = min(sm.topk[d], kmax);
            if (k <= 0) {
                nd = d;
                break;
            }
            const int start = n;
            bool full = false;
            for (int par = frontier_lo; par < frontier_hi && !full; ++par) {
                for (int c = 0; c < k; ++c) {
                    if (n >= cap) {
                        overflow = true;
                        full = true;
                        break;
                    }
                    sm.parents[n] = par;
                    sm.depths[n] = d + 2;
                    sm.cand[n] = c;
                    ++n;
                    if (n >= budget) {
                        full = true;
                        break;
                    }
                }
            }
            frontier_lo = start;
            frontier_hi = n;
            if (frontier_hi == frontier_lo || n >= budget) {
                nd = d + 1;
                break;
            }
        }
        sm.n_depth = nd;
        sm.n_nodes = n;
        int ni = 0;
        for (int i = 0; i < n; ++i) sm.rank[i] = -1;
        for (int i = 1; i < n; ++i) sm.rank[sm.parents[i]] = 0;
        for (int i = 0; i < n; ++i)
            if (sm.rank[i] == 0) sm.rank[i] = ni++, internal_out[ni - 1] = i;
        sm.n_internal = ni;
        for (int i = 0; i < n; ++i) {
            for (int w = 0; w < 4; ++w) sm.anc[i][w] = i > 0 ? sm.anc[sm.parents[i]][w] : 0u;
            sm.anc[i][i >> 5] |= 1u << (i & 31);
        }
        plan_out[0] = sm.budget;
        plan_out[1] = nd;
        for (int d = 0; d < FG_MAX_DEPTHS; ++d) plan_out[2 + d] = d < nd ? sm.topk[d] : 0;
        plan_out[10] = n;
        plan_out[11] = ni;
        plan_out[12] = overflow ? 1 : 0;
        for (int d = 13; d < 16; ++d) plan_out[d] = 0;
    }
    __syncthreads();
    const int n = sm.n_nodes, ni = sm.n_internal;
    for (int i = tid; i < nmax; i += kTreeThreads) {
        const bool valid = i < n;
        parents_out[i] = valid ? sm.parents[i] : -2;
        depths_out[i] = valid ? sm.depths[i] : 1;
        for (int w = 0; w < 4; ++w)
            anc_out[i * 4 + w] = valid ? sm.anc[i][w] : (((i >> 5) == w) ? (1u << (i & 31)) : 0u);
        if (i >= ni) internal_out[i] = -1;
    }
    for (int64_t e = tid; e < (int64_t)B * nmax; e += kTreeThreads) {
        const int b = (int)(e / nmax), i = (int)(e % nmax);
        if (i < n) {
            const int d = sm.depths[i];
            tokens[e] = i == 0 ? root[b] : cand_idx[((int64_t)(d - 2) * B + b) * kmax + sm.cand[i]];
            positions[e] = row_len[b] + d - 1;
            slot[e] = sm.rank[i] >= 0 ? b * ni + sm.rank[i] : -1;
        } else {
            tokens[e] = 0;
            positions[e] = 0;
            slot[e] = -1;
        }
    }
}

}  // namespace fg

using namespace fg;

extern "C" fg_status fg_build_tree(const fg_plan_params* plan, const int32_t* root, const int32_t* cand_idx,
                                   const float* cand_val, const float* head_max, const float* head_lse,
                                   int32_t n_heads, int32_t kmax, int32_t B, int32_t nmax, int32_t logits_dtype,
                                   const int32_t* row_len, int32_t* tokens, int32_t* positions, int32_t* slot,
                                   int32_t* parents, int32_t* depths, uint32_t* anc_bits, int32_t* internal,
                                   int32_t* plan_out, void* stream) {
    if (!plan || !root || !row_len || !tokens || !positions || !slot || !parents || !depths || !anc_bits ||
        !internal || !plan_out)
        return FG_EINVAL;
    if (B <= 0 || nmax <= 0) return FG_EINVAL;
    if (nmax > FG_MAX_TREE_NODES || n_heads > FG_MAX_DEPTHS || kmax > FG_MAX_TOPK) return FG_ECAPACITY;
    if (n_heads > 0 && (!cand_idx || kmax <= 0)) return FG_EINVAL;
    if (plan->adaptive && (B > kSortCap || !cand_val || !head_max || !head_lse)) return plan->adaptive && B > kSortCap ? FG_ECAPACITY : FG_EINVAL;
    if (plan->n_fixed > FG_MAX_DEPTHS || plan->n_min > FG_MAX_DEPTHS) return FG_ECAPACITY;
    build_tree_kernel<<<1, kTreeThreads, 0, (cudaStream_t)stream>>>(
        *plan, root, cand_idx, cand_val, head_max, head_lse, n_heads, kmax, B, nmax, logits_dtype, row_len, tokens,
        positions, slot, parents, depths, anc_bits, internal, plan_out);
    return launch_status();
}

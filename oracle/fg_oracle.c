/*
 * fg_oracle.c -- CPU oracle for the MEDUSA tree-verify hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the parity tests,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg compare the CUDA
 * kernels against.  The product library (libfgb200.so) never links, loads or
 * calls it, and nothing here is a fallback for the GPU path.
 *
 * What it restates (reference = ihbkaiser/ss-GRPO, paths inside that project):
 *   - exact_target acceptance walk: flashgrpo_b200/decoding/acceptance.py:183-267
 *     (single-row form :133-180), with the post-accept clip / EOS / pending
 *     correction rules of flashgrpo_b200/decoding/flash_medusa_decoder.py:2289-2343.
 *   - extract_path KV compaction: flashgrpo_b200/decoding/kv_extraction.py:34-84
 *     (path index :34-51, gather then copy :54-84) on per-row lengths.
 *   - dense MEDUSA tree expansion: flashgrpo_b200/decoding/medusa_tree.py:758-799.
 *   - stable top-k (value descending, index ascending) replacing torch.topk at
 *     medusa_tree.py:767, whose tie order torch leaves unspecified.
 *
 * The sampler is the one piece with no counterpart in the reference: the
 * reference draws with torch.multinomial (acceptance.py:56-60).  Both this
 * oracle and the CUDA kernels implement the same written specification
 * ("fg-icdf-v1", below) independently, so a supplied uniform maps to the same
 * token on both sides, bit for bit:
 *
 *   u        = (philox4x32_10(ctr, key).x >> 8) * 2^-24           in [0, 1-2^-24]
 *              Philox4x32-10 as published by Salmon, Moraes, Dror and Shaw,
 *              "Parallel random numbers: as easy as 1, 2, 3" (SC'11).
 *   x_i      = float(logit_i) / T        (IEEE division; only when T > 0)
 *   m        = max_i x_i
 *   e_i      = fg_exp(x_i - m)           (own exp, see fgo_exp)
 *   lanes    = 512 contiguous chunks of C = roundup8(ceil(V / 512)) entries
 *   c_i      = left-to-right fp32 prefix sum of e inside the chunk of i
 *   s_t      = c at the chunk's last entry (0 for empty chunks)
 *   P_0 = 0, P_{t+1} = P_t + s_t         (sequential over lanes), S = P_512
 *   target   = u * S
 *   t*       = first lane with P_{t+1} > target
 *   token    = first i in chunk t* with P_{t*} + c_i > target
 *   greedy (do_sample == 0 or T == 0): first index of the maximum logit,
 *   matching torch.argmax (acceptance.py:43-44).
 *
 * Nucleus variant "fg-icdf-v1n" (0 < top_p < 1), the kept set of
 * logits_to_probs / sample_from_logits (acceptance.py:7-31, 63-124) stated on
 * exact integer masses so that any summation order gives the same result:
 *   q_i      = trunc(e_i * 2^40)                  (uint64)
 *   Z        = sum q_i,  P = trunc(double(top_p) * double(Z))
 *   key_i    = order-preserving 32-bit image of x_i (-0 counted as +0)
 *   sorted   = key descending, index ascending
 *   K*       = first sorted position whose running mass exceeds P; S is the
 *              running mass there; kept = sorted positions <= K*
 *   t        = trunc(double(u) * double(S))
 *   token    = first index (ascending) among kept entries whose running kept
 *              mass exceeds t.
 *
 * Top-k variant "fg-icdf-v1k" (0 < top_k < V), the top_k branch of
 * sample_from_logits (acceptance.py:68-79: the top_k sorted candidates, a
 * softmax over them, then the nucleus mask when 0 < top_p < 1), with the
 * same integer masses and order:
 *   K-set    = the first top_k sorted positions; Zk = their summed mass
 *   top_p in (0, 1): P = trunc(double(top_p) * double(Zk)) and K*, S as in
 *              v1n (P < Zk puts K* inside the K-set); otherwise K* = the
 *              last K-set position and S = Zk
 *   kept, t and the token as in v1n.
 * torch.topk's order among equal logits is unspecified; here ties go to the
 * lower index, like every other sorted order of this path.
 *
 * Build: oracle/build_oracle.sh (gcc -O2 -ffp-contract=off, no fast-math).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define FGO_LANES 512

/* ---------------------------------------------------------------- Philox */

static uint32_t fgo_mulhilo(uint32_t a, uint32_t b, uint32_t *hi) {
    uint64_t p = (uint64_t)a * (uint64_t)b;
    *hi = (uint32_t)(p >> 32);
    return (uint32_t)p;
}

/* Philox4x32 with 10 rounds (SC'11 paper, section 3.3): multipliers
 * 0xD2511F53 / 0xCD9E8D57, Weyl key increments 0x9E3779B9 / 0xBB67AE85. */
void fgo_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int r = 0; r < 10; ++r) {
        if (r > 0) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        uint32_t hi0, hi1;
        uint32_t lo0 = fgo_mulhilo(0xD2511F53u, c0, &hi0);
        uint32_t lo1 = fgo_mulhilo(0xCD9E8D57u, c2, &hi1);
        uint32_t n0 = hi1 ^ c1 ^ k0;
        uint32_t n2 = hi0 ^ c3 ^ k1;
        c0 = n0;
        c1 = lo1;
        c2 = n2;
        c3 = lo0;
    }
    out[0] = c0;
    out[1] = c1;
    out[2] = c2;
    out[3] = c3;
}

float fgo_uniform(uint64_t seed, uint32_t seq_id, uint32_t round_idx, uint32_t draw) {
    uint32_t ctr[4] = {seq_id, round_idx, draw, 0u};
    uint32_t key[2] = {(uint32_t)(seed & 0xffffffffu), (uint32_t)(seed >> 32)};
    uint32_t out[4];
    fgo_philox4x32_10(ctr, key, out);
    return (float)(out[0] >> 8) * 0x1p-24f;
}

/* out[r * n_draws + d] = uniform for (seq_ids[r], round_idx, d). */
void fgo_philox_uniforms(uint64_t seed, const int32_t *seq_ids, int32_t n_rows, int32_t round_idx,
                         int32_t n_draws, float *out) {
    for (int r = 0; r < n_rows; ++r)
        for (int d = 0; d < n_draws; ++d)
            out[(int64_t)r * n_draws + d] =
                fgo_uniform(seed, (uint32_t)seq_ids[r], (uint32_t)round_idx, (uint32_t)d);
}

/* ------------------------------------------------------------------- exp */

/* exp for the sampler, written from the textbook method: Cody-Waite range
 * reduction x = n*ln2 + r with ln2 split into a 16-significant-bit head
 * (0x3f317200, so n*head is exact) and the fp32-rounded tail (0x35bfbe8e),
 * then the degree-7 Taylor polynomial of e^r on |r| <= ln2/2 evaluated by
 * Horner with fused multiply-adds (coefficients are fp32(1/k!)), scaled by
 * 2^n through the exponent field.  Inputs below -86 (and NaN) give 0, which
 * keeps every result a normal float. */
float fgo_exp(float x) {
    if (!(x >= -86.0f)) return 0.0f;
    const float log2e = 1.44269502162933349609375f; /* 0x3fb8aa3b */
    const float ln2_hi = 0.693145751953125f;         /* 0x3f317200 */
    const float ln2_lo = 1.42860676533018704503775e-06f; /* 0x35bfbe8e */
    float t = x * log2e;
    float nf = rintf(t);
    int n = (int)nf;
    float r = fmaf(-nf, ln2_hi, x);
    r = fmaf(-nf, ln2_lo, r);
    float p = 1.98412701138295233249664e-04f; /* 1/5040 */
    p = fmaf(p, r, 1.38888892251998186111450e-03f); /* 1/720 */
    p = fmaf(p, r, 8.33333376795053482055664e-03f); /* 1/120 */
    p = fmaf(p, r, 4.16666679084300994873047e-02f); /* 1/24 */
    p = fmaf(p, r, 1.66666671633720397949219e-01f); /* 1/6 */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    union {
        uint32_t u;
        float f;
    } s;
    s.u = (uint32_t)(n + 127) << 23;
    return p * s.f;
}

/* --------------------------------------------------------------- sampler */

int32_t fgo_chunk_len(int32_t V) {
    int32_t c = (V + FGO_LANES - 1) / FGO_LANES;
    return (c + 7) & ~7;
}

static float fgo_scaled(const float *logits, int32_t i, float temperature) {
    float v = logits[i];
    if (temperature > 0.0f) v = v / temperature;
    return v;
}

int32_t fgo_argmax(const float *logits, int32_t V) {
    int32_t best = 0;
    float bv = logits[0];
    for (int32_t i = 1; i < V; ++i) {
        if (logits[i] > bv) {
            bv = logits[i];
            best = i;
        }
    }
    return best;
}

/* fg-icdf-v1 sample of one row (see the header comment). */
int32_t fgo_sample_row(const float *logits, int32_t V, float temperature, int32_t do_sample, float u) {
    if (!do_sample || temperature == 0.0f) return fgo_argmax(logits, V);
    float m = -INFINITY;
    for (int32_t i = 0; i < V; ++i) m = fmaxf(m, fgo_scaled(logits, i, temperature));
    const int32_t C = fgo_chunk_len(V);
    float P[FGO_LANES + 1];
    P[0] = 0.0f;
    for (int t = 0; t < FGO_LANES; ++t) {
        float c = 0.0f;
        int32_t lo = t * C, hi = lo + C < V ? lo + C : V;
        for (int32_t i = lo; i < hi; ++i) c = c + fgo_exp(fgo_scaled(logits, i, temperature) - m);
        P[t + 1] = P[t] + c;
    }
    const float S = P[FGO_LANES];
    const float target = u * S;
    for (int t = 0; t < FGO_LANES; ++t) {
        if (P[t + 1] > target) {
            float c = 0.0f;
            int32_t lo = t * C, hi = lo + C < V ? lo + C : V;
            for (int32_t i = lo; i < hi; ++i) {
                c = c + fgo_exp(fgo_scaled(logits, i, temperature) - m);
                if (P[t] + c > target) return i;
            }
            return -1; /* unreachable by construction */
        }
    }
    return -1; /* S == 0: every logit is NaN or -inf */
}

/* ---------------------------------------------------- nucleus (v1n) draw */

typedef struct {
    uint32_t key;
    int32_t idx;
} fgo_keyed;

static uint32_t fgo_nucleus_key(float x) {
    uint32_t b;
    memcpy(&b, &x, 4);
    if (b == 0x80000000u) b = 0u;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

static int fgo_keyed_cmp(const void *pa, const void *pb) {
    const fgo_keyed *a = (const fgo_keyed *)pa, *b = (const fgo_keyed *)pb;
    if (a->key != b->key) return a->key > b->key ? -1 : 1;
    return a->idx < b->idx ? -1 : (a->idx > b->idx ? 1 : 0);
}

/* The fg-icdf-v1n / v1k boundary of one row by an explicit sort (see the
 * header; top_k outside (0, V) means no top-k cut): fills q[V] and returns
 * the boundary index (-1 if every entry is NaN/-inf), with its key in *tau
 * and the running mass there in *S. */
static int32_t fgo_kept_boundary(const float *logits, int32_t V, float temperature, float top_p, int32_t top_k,
                                 uint64_t *q, uint32_t *tau_out, uint64_t *S_out) {
    float m = -INFINITY;
    for (int32_t i = 0; i < V; ++i) m = fmaxf(m, fgo_scaled(logits, i, temperature));
    if (!(m > -INFINITY)) return -1;
    fgo_keyed *ord = (fgo_keyed *)malloc((size_t)V * sizeof(fgo_keyed));
    if (!ord) return -1;
    for (int32_t i = 0; i < V; ++i) {
        const float x = fgo_scaled(logits, i, temperature);
        const float e = fgo_exp(x - m);
        q[i] = (uint64_t)(e * 1099511627776.0f); /* 2^40, exact scaling; truncation */
        ord[i].key = fgo_nucleus_key(x);
        ord[i].idx = i;
    }
    qsort(ord, (size_t)V, sizeof(fgo_keyed), fgo_keyed_cmp);
    const int32_t klim = (top_k > 0 && top_k < V) ? top_k : V;
    uint64_t Zk = 0;
    for (int32_t k = 0; k < klim; ++k) Zk += q[ord[k].idx];
    int32_t istar = -1;
    if (top_p > 0.0f && top_p < 1.0f) {
        const uint64_t P = (uint64_t)((double)top_p * (double)Zk);
        uint64_t cum = 0;
        for (int32_t k = 0; k < klim; ++k) {
            cum += q[ord[k].idx];
            if (cum > P) {
                *tau_out = ord[k].key;
                istar = ord[k].idx;
                *S_out = cum;
                break;
            }
        }
    } else {
        *tau_out = ord[klim - 1].key;
        istar = ord[klim - 1].idx;
        *S_out = Zk;
    }
    free(ord);
    return istar;
}

/* Kept set of an fg-icdf-v1n / v1k draw (mask[i] = 1 for kept entries). */
int32_t fgo_kept_set(const float *logits, int32_t V, float temperature, float top_p, int32_t top_k, uint8_t *mask) {
    uint64_t *q = (uint64_t *)malloc((size_t)V * sizeof(uint64_t));
    if (!q) return -1;
    uint32_t tau = 0;
    uint64_t S = 0;
    const int32_t istar = fgo_kept_boundary(logits, V, temperature, top_p, top_k, q, &tau, &S);
    for (int32_t i = 0; i < V; ++i) {
        const uint32_t key = fgo_nucleus_key(fgo_scaled(logits, i, temperature));
        mask[i] = (istar >= 0 && (key > tau || (key == tau && i <= istar))) ? 1 : 0;
    }
    free(q);
    return istar;
}

int32_t fgo_nucleus_kept(const float *logits, int32_t V, float temperature, float top_p, uint8_t *mask) {
    return fgo_kept_set(logits, V, temperature, top_p, 0, mask);
}

/* fg-icdf-v1n / v1k sample of one row (see the header). */
int32_t fgo_sample_row_kept(const float *logits, int32_t V, float temperature, float top_p, int32_t top_k, float u) {
    uint64_t *q = (uint64_t *)malloc((size_t)V * sizeof(uint64_t));
    if (!q) return -1;
    uint32_t tau = 0;
    uint64_t S = 0;
    const int32_t istar = fgo_kept_boundary(logits, V, temperature, top_p, top_k, q, &tau, &S);
    int32_t token = -1;
    if (istar >= 0) {
        const uint64_t t = (uint64_t)((double)u * (double)S);
        uint64_t run = 0;
        for (int32_t i = 0; i < V; ++i) {
            const uint32_t key = fgo_nucleus_key(fgo_scaled(logits, i, temperature));
            if (key > tau || (key == tau && i <= istar)) {
                run += q[i];
                if (run > t) {
                    token = i;
                    break;
                }
            }
        }
    }
    free(q);
    return token;
}

/* Dispatch: greedy, fg-icdf-v1 (no top-k cut, top_p outside (0, 1)),
 * fg-icdf-v1n (top_p in (0, 1)) or fg-icdf-v1k (0 < top_k < V). */
int32_t fgo_sample_row_pk(const float *logits, int32_t V, float temperature, int32_t do_sample, float top_p,
                          int32_t top_k, float u) {
    if (!do_sample || temperature == 0.0f) return fgo_argmax(logits, V);
    if ((top_p > 0.0f && top_p < 1.0f) || (top_k > 0 && top_k < V))
        return fgo_sample_row_kept(logits, V, temperature, top_p, top_k, u);
    return fgo_sample_row(logits, V, temperature, do_sample, u);
}

void fgo_sample_rows(const float *logits, int64_t row_stride, int32_t V, int32_t n_rows, const float *uniforms,
                     int32_t do_sample, float temperature, float top_p, int32_t top_k, int32_t *out) {
    for (int32_t r = 0; r < n_rows; ++r)
        out[r] = fgo_sample_row_pk(logits + (int64_t)r * row_stride, V, temperature, do_sample, top_p, top_k,
                                   uniforms[r]);
}

/* ------------------------------------------------------- acceptance walk */

/* Restates exact_accept_paths_batch (acceptance.py:183-267) row by row, then
 * the post-accept rules (flash_medusa_decoder.py:2299-2319):
 *   max_accept = max(1, max_length - row_len); EOS cut; finished flag;
 *   the correction is kept as the next root only when the path was not cut
 *   and the row is not finished.
 * Tree children are the nodes whose parent is the current node, in index
 * (BFS) order, as CandidateTree.__post_init__ builds them (medusa_tree.py:19-23).
 * The walk step d of row b uses uniforms[b * u_stride + d].
 * Returns 0, or -(b+1) when row b visits a parent without a logits slot. */
int32_t fgo_accept_walk(const float *logits, int64_t row_stride, int32_t V, const int32_t *slot,
                        const int32_t *tokens, const int32_t *parents, const int32_t *n_nodes, int32_t nmax,
                        const float *uniforms, int32_t u_stride, int32_t B, int32_t do_sample, float temperature,
                        float top_p, int32_t top_k, int32_t eos_id, int32_t max_length, const int32_t *row_len,
                        int32_t dcap,
                        int32_t *acc_tokens, int32_t *acc_nodes, int32_t *acc_len, int32_t *raw_len,
                        int32_t *correction, int32_t *pending, int32_t *last_node, int32_t *finished) {
    for (int32_t b = 0; b < B; ++b) {
        const int32_t *tk = tokens + (int64_t)b * nmax;
        const int32_t *pa = parents + (int64_t)b * nmax;
        const int32_t *sl = slot + (int64_t)b * nmax;
        const int32_t n = n_nodes[b];
        int32_t *at = acc_tokens + (int64_t)b * dcap;
        int32_t *an = acc_nodes + (int64_t)b * dcap;
        int32_t a = 1, parent = 0, corr = -1, step = 0;
        at[0] = tk[0];
        an[0] = 0;
        for (;;) {
            int32_t first_child = -1;
            for (int32_t j = 1; j < n; ++j)
                if (pa[j] == parent) {
                    first_child = j;
                    break;
                }
            if (first_child < 0) break;
            const int32_t s = sl[parent];
            if (s < 0) return -(b + 1);
            const int32_t sampled = fgo_sample_row_pk(logits + (int64_t)s * row_stride, V, temperature, do_sample,
                                                      top_p, top_k, uniforms[(int64_t)b * u_stride + step]);
            ++step;
            int32_t match = -1;
            for (int32_t j = first_child; j < n; ++j)
                if (pa[j] == parent && tk[j] == sampled) {
                    match = j;
                    break;
                }
            if (match < 0) {
                corr = sampled;
                break;
            }
            if (a < dcap) {
                at[a] = sampled;
                an[a] = match;
            }
            ++a;
            parent = match;
        }
        const int32_t raw = a;
        int32_t max_accept = max_length - row_len[b];
        if (max_accept < 1) max_accept = 1;
        if (a > max_accept) a = max_accept;
        int32_t eos_seen = 0;
        for (int32_t p = 0; p < a; ++p)
            if (at[p] == eos_id) {
                a = p + 1;
                eos_seen = 1;
                break;
            }
        const int32_t fin = eos_seen || (row_len[b] + a >= max_length);
        acc_len[b] = a;
        raw_len[b] = raw;
        correction[b] = corr;
        pending[b] = (corr >= 0 && a == raw && !fin) ? corr : -1;
        last_node[b] = an[a - 1];
        finished[b] = fin;
        for (int32_t p = a; p < dcap; ++p) {
            at[p] = -1;
            an[p] = -1;
        }
    }
    return 0;
}

/* --------------------------------------------------------- KV compaction */

/* Per row b, per layer, per kv head: the accepted node path (acc_nodes) is
 * moved from cache slots row_len[b] + node to row_len[b] + j, j < acc_len[b].
 * All path entries of one (layer, row, head) are read before any is written,
 * which is the in-place compaction of kv_extraction.py:70-84 (gather into a
 * temporary, then copy).  cache layout per layer: [B, Hkv, cap, D] with the
 * given element strides; elem_bytes is 2 (bf16/f16) or 4 (f32). */
void fgo_extract_path(uint8_t *const *k_layers, uint8_t *const *v_layers, int32_t n_layers, int32_t B,
                      int32_t Hkv, int32_t D, int64_t stride_b, int64_t stride_h, int64_t stride_s,
                      int32_t elem_bytes, const int32_t *row_len, const int32_t *acc_nodes, const int32_t *acc_len,
                      int32_t dcap) {
    const int64_t vec = (int64_t)D * elem_bytes;
    uint8_t *tmp = (uint8_t *)malloc((size_t)(vec * (dcap > 0 ? dcap : 1)));
    for (int32_t l = 0; l < n_layers; ++l)
        for (int kv = 0; kv < 2; ++kv) {
            uint8_t *base = kv == 0 ? k_layers[l] : v_layers[l];
            for (int32_t b = 0; b < B; ++b)
                for (int32_t h = 0; h < Hkv; ++h) {
                    uint8_t *row = base + (b * stride_b + h * stride_h) * elem_bytes;
                    const int32_t a = acc_len[b];
                    for (int32_t j = 0; j < a; ++j)
                        memcpy(tmp + j * vec, row + (int64_t)(row_len[b] + acc_nodes[(int64_t)b * dcap + j]) * stride_s * elem_bytes,
                               (size_t)vec);
                    for (int32_t j = 0; j < a; ++j)
                        memcpy(row + (int64_t)(row_len[b] + j) * stride_s * elem_bytes, tmp + j * vec, (size_t)vec);
                }
        }
    free(tmp);
}

/* ------------------------------------------------------- dense tree build */

/* Stable top-k of one row: value descending, then index ascending. */
void fgo_topk_stable(const float *row, int32_t V, int32_t k, int32_t *out_idx, float *out_val) {
    for (int32_t j = 0; j < k; ++j) {
        out_idx[j] = -1;
        out_val[j] = -INFINITY;
    }
    for (int32_t i = 0; i < V; ++i) {
        const float v = row[i];
        int32_t pos = k;
        while (pos > 0 && (out_idx[pos - 1] < 0 || v > out_val[pos - 1])) --pos;
        if (pos >= k) continue;
        for (int32_t j = k - 1; j > pos; --j) {
            out_idx[j] = out_idx[j - 1];
            out_val[j] = out_val[j - 1];
        }
        out_idx[pos] = i;
        out_val[pos] = v;
    }
}

/* Restates build_batch_trees (medusa_tree.py:758-799): BFS expansion where
 * every parent at depth d receives the same k_d candidates of head d,
 * truncated at the node budget.  cand_idx is [n_depth][B][kmax].
 * Writes tokens/parents/depths [B][nmax]; returns nothing; n_nodes[b]. */
void fgo_build_dense_trees(const int32_t *root, const int32_t *cand_idx, int32_t kmax, const int32_t *topk_by_depth,
                           int32_t n_depth, int32_t budget, int32_t B, int32_t nmax, int32_t *tokens,
                           int32_t *parents, int32_t *depths, int32_t *n_nodes) {
    int32_t *cur = (int32_t *)malloc(sizeof(int32_t) * (size_t)(nmax + 1));
    int32_t *nxt = (int32_t *)malloc(sizeof(int32_t) * (size_t)(nmax + 1));
    for (int32_t b = 0; b < B; ++b) {
        int32_t *tk = tokens + (int64_t)b * nmax, *pa = parents + (int64_t)b * nmax, *dp = depths + (int64_t)b * nmax;
        int32_t n = 1, ncur = 1, nnxt;
        tk[0] = root[b];
        pa[0] = -1;
        dp[0] = 1;
        cur[0] = 0;
        for (int32_t d = 0; d < n_depth; ++d) {
            const int32_t k = topk_by_depth[d];
            if (k <= 0) break;
            nnxt = 0;
            const int32_t *cands = cand_idx + ((int64_t)d * B + b) * kmax;
            for (int32_t pi = 0; pi < ncur; ++pi) {
                for (int32_t c = 0; c < k; ++c) {
                    tk[n] = cands[c];
                    pa[n] = cur[pi];
                    dp[n] = d + 2;
                    nxt[nnxt++] = n;
                    ++n;
                    if (n >= budget) break;
                }
                if (n >= budget) break;
            }
            int32_t *sw = cur;
            cur = nxt;
            nxt = sw;
            ncur = nnxt;
            if (ncur == 0 || n >= budget) break;
        }
        n_nodes[b] = n;
        for (int32_t j = n; j < nmax; ++j) {
            tk[j] = -1;
            pa[j] = -2;
            dp[j] = 1;
        }
    }
    free(cur);
    free(nxt);
}

// fg_nucleus.cuh -- block-wide nucleus (top-p) draw, "fg-icdf-v1n".
//
// The reference's nucleus sampler (sample_from_logits / logits_to_probs,
// flashgrpo_b200/decoding/acceptance.py:7-31, 63-124) sorts the probabilities
// in descending order, keeps the sorted prefix up to and including the first
// position whose cumulative probability exceeds top_p, and draws from the kept
// weights with torch.multinomial.  fg-icdf-v1n states the same rule on exact
// integers, so a GPU reduction in any order and the CPU checker agree bit for
// bit:
//
//   x_i  = logit_i / T (IEEE), m = max x_i, as in fg-icdf-v1
//   q_i  = trunc(fg_exp(x_i - m) * 2^40)            uint64, q <= 2^40
//   Z    = sum q_i,  P = trunc(double(top_p) * double(Z))
//   key  = order-preserving 32-bit image of x (-0 folded into +0); the sorted
//          order is key descending, index ascending
//   K*   = first sorted position whose inclusive cumulative mass exceeds P;
//          its key tau, index i*, and the cumulative mass S there
//   kept = { key > tau } + { key == tau, index <= i* }
//   t    = trunc(double(u) * double(S))
//   token = first index i (ascending) among kept entries whose running kept
//          mass exceeds t
//
// The kept set is the reference's; the draw maps u to a kept token through
// index order instead of sorted order, which gives every kept token the same
// probability q_i / S without a second search.  K* is found without sorting:
// a 4-level radix select over the keys (8-bit digits, exact integer bucket
// masses), then an index-ordered scan of the boundary key's entries.
//
// Top-k variant "fg-icdf-v1k" (0 < top_k < V; the top_k branch of
// sample_from_logits, acceptance.py:68-79): the K-set is the first top_k
// sorted positions, found by the same radix select on counts instead of
// masses; Zk = its mass; with 0 < top_p < 1, P = trunc(double(top_p) *
// double(Zk)) and K* as above (P < Zk puts K* inside the K-set), otherwise
// K* = the K-set's last position and S = Zk; the draw as above.
#pragma once

#include "fg_sampler.cuh"

namespace fg {

struct NucleusSmem {
    unsigned long long hist[256];
    unsigned long long part[FG_SAMPLE_LANES + 1];
    unsigned long long red[FG_SAMPLE_LANES / 32];
    unsigned long long base;   // mass of entries sorted before the current bucket
    unsigned long long S;      // cumulative mass at the boundary
    uint32_t prefix;           // selected key bits so far
    int32_t istar;             // boundary index
    int32_t result;
};

__device__ __forceinline__ uint32_t nucleus_key(float x) {
    uint32_t b = __float_as_uint(x);
    b = (b == 0x80000000u) ? 0u : b;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ unsigned long long nucleus_q(float x_scaled, float m) {
    return __float2ull_rz(__fmul_rn(fg_exp(__fsub_rn(x_scaled, m)), 1099511627776.0f));  // 2^40
}

// Adds q to h[digit] for the active lanes of a warp; every lane of the warp
// calls it.  Lanes with equal digits are summed first (two 20-bit halves, so
// the 32-bit warp reductions cannot overflow), then one 64-bit atomic each.
__device__ __forceinline__ void nucleus_hist_add(unsigned long long* h, uint32_t digit, unsigned long long q,
                                                 bool active) {
    const unsigned act = __ballot_sync(0xffffffffu, active);
    if (!active) return;
    const unsigned peers = __match_any_sync(act, digit);
    const uint32_t shi = __reduce_add_sync(peers, (uint32_t)(q >> 20));
    const uint32_t slo = __reduce_add_sync(peers, (uint32_t)(q & 0xFFFFFull));
    if ((int)(__ffs(peers) - 1) == (int)(threadIdx.x & 31))
        atomicAdd(&h[digit], ((unsigned long long)shi << 20) + (unsigned long long)slo);
}

__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long v, NucleusSmem& ns) {
    const int tid = threadIdx.x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((tid & 31) == 0) ns.red[tid >> 5] = v;
    __syncthreads();
    unsigned long long t = 0;
#pragma unroll
    for (int w = 0; w < FG_SAMPLE_LANES / 32; ++w) t += ns.red[w];
    __syncthreads();
    return t;
}

// One radix level: histogram of digit (key >> shift) & 255 over the entries
// whose key bits above the digit equal `prefix` (all entries when shift = 24).
// kCount: each entry weighs 1 instead of its mass q.
template <typename T, bool kCount = false>
__device__ __forceinline__ unsigned long long nucleus_level(const T* row, int32_t V, float temperature, float m,
                                                            int shift, uint32_t prefix, bool with_total,
                                                            NucleusSmem& ns) {
    const int tid = threadIdx.x;
    for (int i = tid; i < 256; i += FG_SAMPLE_LANES) ns.hist[i] = 0ull;
    __syncthreads();
    unsigned long long tot = 0;
    // uniform trip count across the block so every warp reaches the warp
    // intrinsics of nucleus_hist_add together
    for (int32_t base = 0; base < V; base += FG_SAMPLE_LANES) {
        const int32_t i = base + tid;
        bool act = i < V;
        float x = 0.0f;
        if (act) x = scale_t(to_f<T>(row[i]), temperature);
        const uint32_t key = nucleus_key(x);
        const uint32_t above_bits = shift == 24 ? 0u : (key >> (shift + 8));  // shift + 8 <= 24 here
        act = act && above_bits == prefix;
        const unsigned long long q = act ? (kCount ? 1ull : nucleus_q(x, m)) : 0ull;
        if (with_total) tot += q;
        nucleus_hist_add(ns.hist, (key >> shift) & 255u, q, act);
    }
    __syncthreads();
    return tot;
}

// Thread 0: the bucket (scanning digits from high to low) in which the
// cumulative mass, starting at ns.base, first exceeds thr.
__device__ __forceinline__ void nucleus_pick(unsigned long long thr, int shift, NucleusSmem& ns) {
    if (threadIdx.x == 0) {
        unsigned long long acc = ns.base;
        int sel = 0;
        for (int d = 255; d >= 0; --d) {
            if (acc + ns.hist[d] > thr) {
                sel = d;
                break;
            }
            acc += ns.hist[d];
        }
        ns.base = acc;
        ns.prefix = (shift == 24) ? (uint32_t)sel : ((ns.prefix << 8) | (uint32_t)sel);
    }
    __syncthreads();
}

// Index-ordered pass over thread chunks: each thread sums f(i) over its
// contiguous chunk; thread 0 turns the sums into exclusive prefixes.
template <typename T, typename F>
__device__ __forceinline__ void nucleus_chunk_sums(const T* row, int32_t V, int32_t C, F f, NucleusSmem& ns) {
    const int tid = threadIdx.x;
    const int32_t lo = min(tid * C, V), hi = min(lo + C, V);
    unsigned long long c = 0;
    for (int32_t i = lo; i < hi; ++i) c += f(i);
    ns.part[tid + 1] = c;
    __syncthreads();
    if (tid == 0) {
        unsigned long long acc = 0;
        ns.part[0] = 0;
        for (int t = 0; t < FG_SAMPLE_LANES; ++t) {
            acc += ns.part[t + 1];
            ns.part[t + 1] = acc;
        }
    }
    __syncthreads();
}

struct SortedPick {
    int32_t idx;               // -1: the weights never exceed the threshold
    uint32_t key;
    unsigned long long weight; // running weight at idx
};

// Finishes a sorted-order selection whose first radix level the caller has
// run: the first sorted position (key descending, index ascending) at which
// the running weight (mass q, or 1 with kCount) exceeds thr.
template <typename T, bool kCount>
__device__ __forceinline__ SortedPick sorted_select_finish(const T* row, int32_t V, float temperature, float m,
                                                           unsigned long long thr, NucleusSmem& ns) {
    const int tid = threadIdx.x;
    nucleus_pick(thr, 24, ns);
    for (int shift = 16; shift >= 0; shift -= 8) {
        const uint32_t prefix = ns.prefix;
        nucleus_level<T, kCount>(row, V, temperature, m, shift, prefix, false, ns);
        nucleus_pick(thr, shift, ns);
    }
    const uint32_t key_sel = ns.prefix;
    const unsigned long long above = ns.base;  // weight of keys > key_sel
    // boundary entry: index order inside the key == key_sel group
    const int32_t C = sample_chunk_len(V);
    auto tie_w = [&](int32_t i) -> unsigned long long {
        const float x = scale_t(to_f<T>(row[i]), temperature);
        return nucleus_key(x) == key_sel ? (kCount ? 1ull : nucleus_q(x, m)) : 0ull;
    };
    nucleus_chunk_sums<T>(row, V, C, tie_w, ns);
    if (tid == 0) ns.istar = -1;
    __syncthreads();
    {
        const unsigned long long p0 = above + ns.part[tid], p1 = above + ns.part[tid + 1];
        if (p0 <= thr && thr < p1) {
            const int32_t lo = min(tid * C, V), hi = min(lo + C, V);
            unsigned long long acc = p0;
            for (int32_t i = lo; i < hi; ++i) {
                acc += tie_w(i);
                if (acc > thr) {
                    ns.istar = i;
                    ns.S = acc;
                    break;
                }
            }
        }
    }
    __syncthreads();
    const SortedPick r{ns.istar, key_sel, ns.S};
    __syncthreads();
    return r;
}

// fg-icdf-v1n / v1k draw (0 < top_p < 1 or 0 < top_k < V; T > 0, do_sample);
// returns -1 only when every entry is NaN or -inf.
template <typename T>
__device__ int32_t block_sample_kept(const T* row, int32_t V, float temperature, float top_p, int32_t top_k,
                                     float u, SampleSmem& sm, NucleusSmem& ns) {
    const int tid = threadIdx.x;
    float bv;
    int32_t bi;
    row_max<T>(row, V, bv, bi);
    block_best(bv, bi, sm);
    const float m = scale_t(sm.red[0], temperature);
    __syncthreads();
    if (!(m > -INFINITY)) return -1;
    const bool cut_k = top_k > 0 && top_k < V;
    const bool cut_p = top_p > 0.0f && top_p < 1.0f;
    uint32_t tau = 0;
    int32_t istar = -1;
    unsigned long long S = 0;
    if (cut_k) {
        // the K-set: sorted positions 0 .. top_k - 1, by a count selection
        if (tid == 0) ns.base = 0ull;
        nucleus_level<T, true>(row, V, temperature, m, 24, 0u, false, ns);
        const SortedPick kp =
            sorted_select_finish<T, true>(row, V, temperature, m, (unsigned long long)(top_k - 1), ns);
        if (kp.idx < 0) return -1;
        const uint32_t tau_k = kp.key;
        const int32_t i_k = kp.idx;
        // Zk: the K-set's mass
        unsigned long long zpart = 0;
        for (int32_t i = tid; i < V; i += FG_SAMPLE_LANES) {
            const float x = scale_t(to_f<T>(row[i]), temperature);
            const uint32_t k = nucleus_key(x);
            if (k > tau_k || (k == tau_k && i <= i_k)) zpart += nucleus_q(x, m);
        }
        const unsigned long long Zk = block_sum_u64(zpart, ns);
        if (cut_p) {
            const unsigned long long P = __double2ull_rz(__dmul_rn((double)top_p, __ull2double_rn(Zk)));
            if (tid == 0) ns.base = 0ull;
            nucleus_level<T>(row, V, temperature, m, 24, 0u, false, ns);
            const SortedPick pp = sorted_select_finish<T, false>(row, V, temperature, m, P, ns);
            istar = pp.idx;
            tau = pp.key;
            S = pp.weight;
        } else {
            tau = tau_k;
            istar = i_k;
            S = Zk;
        }
    } else {
        // level 1 with the total mass
        if (tid == 0) ns.base = 0ull;
        const unsigned long long z_part = nucleus_level<T>(row, V, temperature, m, 24, 0u, true, ns);
        const unsigned long long Z = block_sum_u64(z_part, ns);
        const unsigned long long P = __double2ull_rz(__dmul_rn((double)top_p, __ull2double_rn(Z)));
        const SortedPick pp = sorted_select_finish<T, false>(row, V, temperature, m, P, ns);
        istar = pp.idx;
        tau = pp.key;
        S = pp.weight;
    }
    if (istar < 0) return -1;
    // the draw: index order over the kept entries
    const int32_t C = sample_chunk_len(V);
    const unsigned long long t = __double2ull_rz(__dmul_rn((double)u, __ull2double_rn(S)));
    auto kept_q = [&](int32_t i) -> unsigned long long {
        const float x = scale_t(to_f<T>(row[i]), temperature);
        const uint32_t k = nucleus_key(x);
        return (k > tau || (k == tau && i <= istar)) ? nucleus_q(x, m) : 0ull;
    };
    nucleus_chunk_sums<T>(row, V, C, kept_q, ns);
    if (tid == 0) ns.result = -1;
    __syncthreads();
    if (ns.part[tid] <= t && t < ns.part[tid + 1]) {
        const int32_t lo = min(tid * C, V), hi = min(lo + C, V);
        unsigned long long acc = ns.part[tid];
        for (int32_t i = lo; i < hi; ++i) {
            acc += kept_q(i);
            if (acc > t) {
                ns.result = i;
                break;
            }
        }
    }
    __syncthreads();
    const int32_t r = ns.result;
    __syncthreads();
    return r;
}

// True when a draw with these knobs takes the kept-set form (v1n / v1k).
__host__ __device__ __forceinline__ bool sample_cuts(int32_t do_sample, float temperature, float top_p,
                                                     int32_t top_k, int32_t V) {
    return do_sample != 0 && temperature != 0.0f && ((top_p > 0.0f && top_p < 1.0f) || (top_k > 0 && top_k < V));
}

}  // namespace fg

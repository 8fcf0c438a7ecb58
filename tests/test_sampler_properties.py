"""Properties of the fg-icdf-v1n / v1k kept sets and draws (CPU oracle).

The golden fixtures pin the kept sets to the reference on seeded rows; these
tests check the rules themselves on many generated rows, including ties:
the kept set is a prefix of the sorted order (value descending, index
ascending), holds at most top_k entries, and is the shortest prefix whose
renormalised mass exceeds top_p; every draw lands in it.
"""
from __future__ import annotations

import numpy as np
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from oracle import native


def _sorted_order(x: np.ndarray) -> np.ndarray:
    return np.lexsort((np.arange(x.size), -x.astype(np.float64)))


rows = st.integers(min_value=2, max_value=400).flatmap(
    lambda n: st.tuples(
        st.just(n),
        st.integers(min_value=0, max_value=2 ** 31 - 1),
        st.sampled_from([0.05, 0.5, 2.0, 6.0]),
        st.booleans(),
    ))


@settings(max_examples=120, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(row=rows, top_k=st.integers(min_value=0, max_value=500), top_p=st.sampled_from([1.0, 0.99, 0.9, 0.5, 0.1]),
       temperature=st.sampled_from([1.0, 0.7, 1.5]))
def test_kept_set_is_the_rule_prefix(row, top_k, top_p, temperature):
    n, seed, scale, ties = row
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(n) * scale).astype(np.float32)
    if ties:
        x = np.round(x).astype(np.float32)
    keep = native.kept_set(x, temperature, top_p, top_k)
    xs32 = x / np.float32(temperature)  # the order is the scaled values' (IEEE division, as the sampler)
    order = _sorted_order(xs32)
    k = int(keep.sum())
    assert k >= 1
    # a prefix of the sorted order
    assert keep[order[:k]].all() and not keep[order[k:]].any()
    # at most top_k entries when top_k cuts
    if 0 < top_k < n:
        assert k <= top_k
    # the shortest prefix whose renormalised mass exceeds top_p (float64
    # restatement of the integer rule; the boundary test skips near-ties)
    if 0.0 < top_p < 1.0:
        lim = top_k if 0 < top_k < n else n
        xs = xs32.astype(np.float64)[order[:lim]]
        p = np.exp(xs - xs.max())
        cum = np.cumsum(p) / p.sum()
        want = int(np.argmax(cum > top_p)) + 1
        margin = min(abs(cum[want - 1] - top_p), abs(cum[want - 2] - top_p) if want >= 2 else 1.0)
        if margin > 1e-5:
            assert k == want
    elif 0 < top_k < n:
        assert k == top_k


@settings(max_examples=40, deadline=None)
@given(seed=st.integers(min_value=0, max_value=2 ** 31 - 1), top_k=st.integers(min_value=1, max_value=64),
       top_p=st.sampled_from([1.0, 0.9, 0.5]))
def test_draws_land_in_the_kept_set(seed, top_k, top_p):
    rng = np.random.default_rng(seed)
    V = 257
    x = (rng.standard_normal(V) * 3.0).astype(np.float32)
    keep = native.kept_set(x, 1.0, top_p, top_k)
    u = native.philox_uniforms(seed & 0xFFFF, np.arange(200), 1, 1)[:, 0]
    s = native.sample_rows(np.broadcast_to(x, (200, V)).copy(), u, top_p=top_p, top_k=top_k)
    assert keep[s].all()
    # the extremes of u hit the first and the last kept index (index order)
    lo = native.sample_rows(x, [0.0], top_p=top_p, top_k=top_k)[0]
    hi = native.sample_rows(x, [1.0 - 2 ** -24], top_p=top_p, top_k=top_k)[0]
    kept_idx = np.nonzero(keep)[0]
    assert lo == kept_idx[0]
    assert hi in kept_idx

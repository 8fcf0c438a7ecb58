"""Pin the CPU oracle to the reference before it is trusted as a checker.

Each test restates a known-answer test of the reference's own suite
(flashgrpo_b200/tests/*) or compares the oracle with fixtures that
tests/golden/make_golden.py produced by running the reference itself.
"""
from __future__ import annotations

import json
import math

import numpy as np
import pytest
import torch

from conftest import compare_stats
from oracle import native
from oracle import reference_path as rp


# ---------------------------------------------------------------- sampler
def test_philox_matches_published_known_answers():
    # Random123 known-answer vectors for philox4x32_10 (Salmon et al., SC'11).
    assert native.philox4x32_10([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert native.philox4x32_10([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert native.philox4x32_10([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0]) == [
        0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_uniform_range_and_independence():
    u = native.philox_uniforms(7, np.arange(4096), 3, 4)
    assert u.min() >= 0.0 and u.max() < 1.0
    assert abs(float(u.mean()) - 0.5) < 0.01
    assert len(np.unique(u)) > 0.99 * u.size


def test_exp_within_one_ulp_of_true_exp():
    xs = np.concatenate([np.linspace(-86, 0, 20001), -np.logspace(-8, 1.9, 2000), [0.0, -1e-30]]).astype(np.float32)
    mine = native.exp_array(xs).astype(np.float64)
    true = np.exp(xs.astype(np.float64))
    ulp = np.spacing(true.astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(mine - true) / ulp) <= 1.0
    assert native.fg_exp(-86.5) == 0.0 and native.fg_exp(float("nan")) == 0.0


def test_sampler_matches_target_distribution():
    # acceptance test :74-93 -- p = [0.6, 0.4], 50 000 draws, error < 0.015
    logits = np.log(np.array([0.6, 0.4], dtype=np.float32))
    u = native.philox_uniforms(456, np.arange(50_000), 0, 1)[:, 0]
    x = np.broadcast_to(logits, (50_000, 2)).copy()
    s = native.sample_rows(x, u)
    freq = np.bincount(s, minlength=2) / s.size
    assert np.max(np.abs(freq - [0.6, 0.4])) < 0.015


def test_sampler_distribution_large_vocab_and_temperature():
    rng = np.random.default_rng(3)
    logits = (rng.standard_normal(1000) * 2).astype(np.float32)
    for temp in (1.0, 0.7):
        p = np.exp(logits.astype(np.float64) / temp)
        p /= p.sum()
        u = native.philox_uniforms(9, np.arange(60_000), 1, 1)[:, 0]
        s = native.sample_rows(np.broadcast_to(logits, (60_000, 1000)).copy(), u, temperature=temp)
        freq = np.bincount(s, minlength=1000) / s.size
        assert np.max(np.abs(freq - p)) < 0.015
        assert np.all(p[np.unique(s)] > 0)


def test_sampler_never_picks_zero_probability_and_greedy_is_first_max():
    x = np.full(700, -1e30, dtype=np.float32)
    x[[5, 399, 650]] = [1.0, 3.0, 3.0]
    s = native.sample_rows(np.broadcast_to(x, (2000, 700)).copy(), np.linspace(0, 0.99999994, 2000, dtype=np.float32))
    assert set(np.unique(s)) <= {5, 399, 650}
    assert native.sample_rows(x, [0.5], do_sample=False)[0] == 399
    assert native.sample_rows(x, [0.5], temperature=0.0)[0] == 399
    # u at the top of its range still lands on a positive-probability entry
    assert native.sample_rows(x, [1.0 - 2 ** -24])[0] in (399, 650)


# ------------------------------------------------------- nucleus (top-p)
def test_nucleus_kept_set_matches_reference(golden_dir):
    # logits_to_probs (acceptance.py:7-31) on 48 seeded rows, 4 vocab sizes,
    # 3 temperatures, top_p in {0.5, 0.8, 0.9, 0.95, 0.99}
    d = np.load(golden_dir / "nucleus.npz")
    compared = 0
    for r in range(d["logits"].shape[0]):
        V = int(d["vocab"][r])
        if d["margin"][r] < 1e-5:  # boundary within fp32 rounding of the reference's cumsum
            continue
        mine = native.nucleus_kept(d["logits"][r, :V], float(d["temperature"][r]), float(d["top_p"][r]))
        assert np.array_equal(mine, d["kept"][r, :V]), r
        compared += 1
    assert compared >= 40


def test_nucleus_sampler_matches_renormalised_kept_distribution():
    rng = np.random.default_rng(11)
    logits = (rng.standard_normal(300) * 2).astype(np.float32)
    for temp, top_p in ((1.0, 0.9), (0.7, 0.5)):
        p = np.exp((logits.astype(np.float64) - logits.max()) / temp)
        p /= p.sum()
        keep = native.nucleus_kept(logits, temp, top_p)
        # the reference rule: sorted prefix through the first cumulative > top_p
        order = np.argsort(-logits, kind="stable")
        k = int(np.argmax(np.cumsum(p[order]) > top_p))
        want = np.zeros(300, dtype=bool)
        want[order[: k + 1]] = True
        assert np.array_equal(keep, want)
        q = np.where(keep, p, 0.0)
        q /= q.sum()
        u = native.philox_uniforms(21, np.arange(60_000), 3, 1)[:, 0]
        s = native.sample_rows(np.broadcast_to(logits, (60_000, 300)).copy(), u, temperature=temp, top_p=top_p)
        assert keep[s].all()
        freq = np.bincount(s, minlength=300) / s.size
        assert np.max(np.abs(freq - q)) < 0.015


def test_nucleus_edges_ties_and_tiny_top_p():
    # bf16-like ties: equal values are ordered by index, the boundary can cut a tie group
    x = np.array([1.0, 2.0, 2.0, 2.0, 0.0, 2.0], dtype=np.float32)
    p = np.exp(x - 2.0) / np.exp(x - 2.0).sum()
    keep = native.nucleus_kept(x, 1.0, 0.5)
    k = int(np.argmax(np.cumsum(p[[1, 2, 3, 5, 0, 4]]) > 0.5))
    assert keep.tolist() == [i in [1, 2, 3, 5, 0, 4][: k + 1] for i in range(6)]
    # a tiny top_p keeps only the first maximum: the draw is the argmax for every u
    u = np.linspace(0, 1 - 2 ** -24, 64, dtype=np.float32)
    assert set(native.sample_rows(np.broadcast_to(x, (64, 6)).copy(), u, top_p=1e-6).tolist()) == {1}
    # top_p outside (0, 1) is fg-icdf-v1; greedy ignores top_p
    y = (np.random.default_rng(2).standard_normal(500)).astype(np.float32)
    uu = native.philox_uniforms(5, np.arange(50), 0, 1)[:, 0]
    rows = np.broadcast_to(y, (50, 500)).copy()
    assert np.array_equal(native.sample_rows(rows, uu, top_p=1.0), native.sample_rows(rows, uu))
    assert native.sample_rows(y, [0.3], do_sample=False, top_p=0.5)[0] == int(np.argmax(y))


# ------------------------------------------------------------ acceptance
def _walk(tokens, parents, logits, slots=None, do_sample=False, u=None, dcap=6, row_len=None, max_length=1 << 30,
          eos=-7):
    tokens = np.atleast_2d(np.asarray(tokens, dtype=np.int32))
    parents = np.atleast_2d(np.asarray(parents, dtype=np.int32))
    B, n = tokens.shape
    n_nodes = np.full(B, n, dtype=np.int32)
    if slots is None:
        slots = np.arange(B * n, dtype=np.int32).reshape(B, n)
    if u is None:
        u = np.zeros((B, 8), dtype=np.float32)
    return native.accept_walk(np.asarray(logits, dtype=np.float32).reshape(-1, np.shape(logits)[-1]), slots, tokens,
                              parents, n_nodes, u, do_sample=do_sample, temperature=1.0, eos_id=eos,
                              max_length=max_length, row_len=np.zeros(B) if row_len is None else row_len, dcap=dcap)


def test_greedy_accepts_only_target_child():
    # acceptance test :40-55
    logits = np.full((3, 16), -10.0, dtype=np.float32)
    logits[0, 7] = 10.0
    r = _walk([5, 7, 9], [-1, 0, 0], logits)
    assert r["acc_tokens"][0, :2].tolist() == [5, 7] and r["acc_nodes"][0, :2].tolist() == [0, 1]
    assert r["acc_len"][0] == 2 and r["correction"][0] == -1


def test_mismatch_returns_correction_token():
    # acceptance test :58-71
    logits = np.full((2, 16), -10.0, dtype=np.float32)
    logits[0, 9] = 10.0
    r = _walk([5, 7], [-1, 0], logits)
    assert r["acc_len"][0] == 1 and r["acc_nodes"][0, 0] == 0 and r["correction"][0] == 9
    assert r["pending"][0] == 9


def test_stochastic_match_or_correction_preserves_target():
    # acceptance test :74-93 through the walk
    n = 50_000
    logits = np.log(np.array([[0.6, 0.4]] * 2, dtype=np.float32))
    u = native.philox_uniforms(456, np.arange(n), 0, 2)
    tokens = np.tile([[2, 0]], (n, 1))
    parents = np.tile([[-1, 0]], (n, 1))
    slots = np.tile([[0, -1]], (n, 1))
    r = native.accept_walk(logits, slots, tokens, parents, np.full(n, 2), u, do_sample=True, temperature=1.0,
                           eos_id=-7, max_length=1 << 30, row_len=np.zeros(n), dcap=3)
    emitted = np.where(r["acc_len"] > 1, r["acc_tokens"][:, 1], r["correction"])
    assert np.all(emitted >= 0)
    freq = np.bincount(emitted, minlength=2) / n
    assert np.max(np.abs(freq - [0.6, 0.4])) < 0.015


def test_packed_internal_logits_match_dense():
    # acceptance test :96-137
    tokens = [[5, 7, 9, 11], [4, 6, 8, 10]]
    parents = [[-1, 0, 0, 1], [-1, 0, 0, 2]]
    dense = np.full((2, 4, 16), -10.0, dtype=np.float32)
    dense[0, 0, 7] = dense[0, 1, 11] = dense[1, 0, 8] = dense[1, 2, 10] = 10.0
    packed = np.stack([dense[0, 0], dense[0, 1], dense[1, 0], dense[1, 2]])
    slots = np.array([[0, 1, -1, -1], [2, -1, 3, -1]], dtype=np.int32)
    d = _walk(tokens, parents, dense.reshape(8, 16))
    p = _walk(tokens, parents, packed, slots=slots)
    for k in ("acc_tokens", "acc_nodes", "acc_len", "correction", "last_node"):
        assert np.array_equal(d[k], p[k]), k
    assert d["acc_tokens"][0, :3].tolist() == [5, 7, 11] and d["acc_tokens"][1, :3].tolist() == [4, 8, 10]


def test_post_accept_clip_eos_and_pending_rules():
    # flash_medusa_decoder.py:2299-2319
    logits = np.full((3, 16), -10.0, dtype=np.float32)
    logits[0, 7] = logits[1, 11] = 10.0
    # full path [5, 7, 11] then leaf: no correction
    r = _walk([5, 7, 11], [-1, 0, 1], logits)
    assert r["acc_len"][0] == 3 and r["pending"][0] == -1 and r["last_node"][0] == 2
    # only one slot left: clip to 1 and finish
    r = _walk([5, 7, 11], [-1, 0, 1], logits, row_len=[9], max_length=10)
    assert r["acc_len"][0] == 1 and r["finished"][0] == 1
    # EOS inside the path cuts it and finishes
    r = _walk([5, 7, 11], [-1, 0, 1], logits, eos=7)
    assert r["acc_len"][0] == 2 and r["finished"][0] == 1 and r["last_node"][0] == 1
    # correction kept only when the path was not cut
    logits2 = np.full((2, 16), -10.0, dtype=np.float32)
    logits2[0, 7] = 10.0
    logits2[1, 3] = 10.0
    r = _walk([5, 7, 9], [-1, 0, 1], logits2)
    assert r["acc_len"][0] == 2 and r["correction"][0] == 3 and r["pending"][0] == 3
    r = _walk([5, 7, 9], [-1, 0, 1], logits2, row_len=[8], max_length=10)
    assert r["acc_len"][0] == 2 and r["finished"][0] == 1 and r["pending"][0] == -1


def test_walk_matches_reference_fixture(golden_dir):
    g = np.load(golden_dir / "accept.npz")
    cases = sorted({k.split("_")[0] for k in g.files})
    assert len(cases) >= 5
    for c in cases:
        V, B, nmax, do_sample = g[c + "_meta"].tolist()
        r = native.accept_walk(g[c + "_logits"], g[c + "_slots"], g[c + "_tokens"], g[c + "_parents"],
                               g[c + "_n_nodes"], g[c + "_uniforms"], do_sample=bool(do_sample),
                               temperature=float(g[c + "_temp"][0]), eos_id=-7, max_length=1 << 30,
                               row_len=np.zeros(B), dcap=5)
        assert np.array_equal(r["acc_tokens"], g[c + "_acc_tokens"]), c
        assert np.array_equal(r["acc_nodes"], g[c + "_acc_nodes"]), c
        assert np.array_equal(r["correction"], g[c + "_correction"]), c
        # the reference returns the raw parent, i.e. the last accepted node
        assert np.array_equal(r["last_node"], g[c + "_parent"]), c


def test_python_walk_equals_c_walk(golden_dir):
    g = np.load(golden_dir / "accept.npz")
    c = "c2"
    V, B, nmax, _ = g[c + "_meta"].tolist()
    tok, par, nn = g[c + "_tokens"], g[c + "_parents"], g[c + "_n_nodes"]
    trees = [rp.Tree(tok[b, :nn[b]].tolist(), par[b, :nn[b]].tolist(), [1] * nn[b]) for b in range(B)]
    U = g[c + "_uniforms"]

    def sampler(rows, seq_ids, round_idx, draw, *, do_sample, temperature):
        return native.sample_rows(rows.numpy(), [U[s, draw - 1] for s in seq_ids], do_sample=do_sample,
                                  temperature=temperature)

    acc, accn, _, corr = rp.accept_walk_batch(trees, torch.from_numpy(g[c + "_logits"]), g[c + "_slots"].tolist(),
                                              sampler, list(range(B)), 0, do_sample=True, temperature=1.0)
    r = native.accept_walk(g[c + "_logits"], g[c + "_slots"], tok, par, nn, U, do_sample=True, temperature=1.0,
                           eos_id=-7, max_length=1 << 30, row_len=np.zeros(B), dcap=5)
    for b in range(B):
        assert r["acc_tokens"][b, : r["acc_len"][b]].tolist() == acc[b]
        assert r["acc_nodes"][b, : r["acc_len"][b]].tolist() == accn[b]
        assert r["correction"][b] == (-1 if corr[b] is None else corr[b])


# ------------------------------------------------------------ extraction
def test_in_place_compaction_matches_copy_path():
    # kv_path_extraction test :14-35 (seed 17): in-place == gather+cat
    torch.manual_seed(17)
    old_len, tree_nodes = 5, 4
    key = torch.randn(2, 2, old_len + tree_nodes, 8)
    value = torch.randn_like(key)
    accepted = [[0, 1, 3], [0, 2]]
    k_np, v_np = key.numpy().copy(), value.numpy().copy()
    acc_nodes = np.array([[0, 1, 3], [0, 2, -1]], dtype=np.int32)
    native.extract_path([k_np], [v_np], [old_len, old_len], acc_nodes, [3, 2])
    for b, path in enumerate(accepted):
        idx = [old_len + n for n in path]
        assert np.array_equal(k_np[b, :, old_len:old_len + len(path)], key.numpy()[b][:, idx])
        assert np.array_equal(v_np[b, :, old_len:old_len + len(path)], value.numpy()[b][:, idx])
        assert np.array_equal(k_np[b, :, :old_len], key.numpy()[b, :, :old_len])


def test_extract_matches_reference_fixture(golden_dir):
    g = np.load(golden_dir / "extract.npz")
    for c in sorted({k.split("_")[0] for k in g.files}):
        B, H, old, n, D, is_bf16 = g[c + "_meta"].tolist()
        paths = g[c + "_paths"]
        lens = (paths >= 0).sum(1).astype(np.int32)
        ks = [g[c + "_k0"].copy(), g[c + "_k1"].copy()]
        vs = [g[c + "_v0"].copy(), g[c + "_v1"].copy()]
        native.extract_path(ks, vs, np.full(B, old), paths, lens)
        for li in range(2):
            rk, rv = g[c + f"_rk{li}"], g[c + f"_rv{li}"]
            assert rk.shape[2] == old + int(g[c + "_max_len"][0])
            for b in range(B):
                a = old + lens[b]
                assert np.array_equal(ks[li][b, :, :a], rk[b, :, :a]), (c, li, b)
                assert np.array_equal(vs[li][b, :, :a], rv[b, :, :a]), (c, li, b)


# ------------------------------------------------------------ trees/masks
def test_mask_allows_only_ancestors():
    # tree_attention_equivalence test :9-20
    t = rp.Tree([1, 2, 3, 4], [-1, 0, 0, 1], [1, 2, 2, 3])
    _, mask, pos, node_mask = rp.tree_attention_inputs([t], torch.ones(1, 5, dtype=torch.long), torch.tensor([5]),
                                                       pad_token_id=0, dtype=torch.float32)
    assert node_mask[0, 3]
    assert mask[0, 0, 3, 5] == 0 and mask[0, 0, 3, 6] == 0 and mask[0, 0, 3, 8] == 0
    assert mask[0, 0, 3, 7] < -1e20
    assert int(pos[0, 3]) == 7


def test_trees_masks_and_slots_match_reference_fixture(golden_dir):
    g = np.load(golden_dir / "trees.npz")
    for p in sorted({k.split("_")[0] for k in g.files}):
        plan_arr = g[p + "_plan"].tolist()
        plan = rp.Plan(plan_arr[0], len(plan_arr) - 1, plan_arr[1:], 0, "x")
        root = g[p + "_root"]
        logits = torch.from_numpy(g[p + "_logits"])
        trees = rp.build_dense_trees(root.tolist(), list(logits), plan)
        nmax = g[p + "_tokens"].shape[1]
        assert np.array_equal(np.array([t.tokens + [-1] * (nmax - t.node_count) for t in trees]), g[p + "_tokens"])
        assert np.array_equal(np.array([t.parents + [-2] * (nmax - t.node_count) for t in trees]), g[p + "_parents"])
        assert np.array_equal(np.array([t.depths + [1] * (nmax - t.node_count) for t in trees]), g[p + "_depths"])
        # the C oracle builds the same trees from stable top-k candidates
        kmax = max(plan.topk_by_depth)
        cand = np.stack([np.stack([native.topk_stable(logits[d, b].numpy(), kmax)[0] for b in range(len(root))])
                         for d in range(plan.active_heads)])
        ct = native.build_dense_trees(root, cand, plan.topk_by_depth, plan.node_budget_per_seq, nmax)
        assert np.array_equal(ct["tokens"], g[p + "_tokens"]) and np.array_equal(ct["parents"], g[p + "_parents"])
        full = torch.from_numpy(g[p + "_full_mask"])
        ids, mask, pos, node_mask = rp.tree_attention_inputs(trees, full, full.sum(-1), pad_token_id=0,
                                                             dtype=torch.float32)
        assert np.array_equal((mask == 0).numpy(), g[p + "_allowed"])
        assert np.array_equal(pos.numpy(), g[p + "_pos"]) and np.array_equal(ids.numpy(), g[p + "_ids"])
        assert np.array_equal(node_mask.numpy(), g[p + "_node_mask"])
        assert np.array_equal(np.array(rp.internal_logit_layout(trees)[2]), g[p + "_slots"])


# ---------------------------------------------------------------- planner
def test_planner_known_answers():
    # test_flashgrpo_smoke.py:20-61
    kw = dict(num_medusa_heads=3, tree_mode="concurrency_aware", min_tree_nodes_per_seq=1, max_tree_depth=4,
              fixed_tree_topk_by_depth=[4, 3, 2])
    small = rp.plan_tree(active_batch_size=1, cpeak_nodes=32, max_tree_nodes_per_seq=16, **kw)
    large = rp.plan_tree(active_batch_size=16, cpeak_nodes=32, max_tree_nodes_per_seq=16, **kw)
    assert small.actual_nodes >= large.actual_nodes
    p = rp.plan_tree(active_batch_size=64, cpeak_nodes=256, max_tree_nodes_per_seq=12, adaptive_tree_enabled=True,
                     adaptive_min_topk_by_depth=[1, 1, 1], **kw)
    assert p.node_budget_per_seq == 4 and p.active_heads == 3
    # config 2: cpeak 1024, B 64, max 16 -> budget 16, plan [4, 2], 13 nodes
    p = rp.plan_tree(active_batch_size=64, cpeak_nodes=1024, max_tree_nodes_per_seq=16, **kw)
    assert (p.node_budget_per_seq, p.topk_by_depth, p.actual_nodes) == (16, [4, 2], 13)


def test_planner_matches_reference_fixture(golden_dir):
    d = json.loads((golden_dir / "planner.json").read_text())
    for mode, bsz, cpeak, mx, depth, topk, adaptive, amin, budget, heads, out_topk, nodes in d["plans"]:
        p = rp.plan_tree(active_batch_size=bsz, num_medusa_heads=4, tree_mode=mode, cpeak_nodes=cpeak,
                         min_tree_nodes_per_seq=1, max_tree_nodes_per_seq=mx, max_tree_depth=depth,
                         fixed_tree_topk_by_depth=topk, adaptive_tree_enabled=adaptive,
                         adaptive_min_topk_by_depth=amin)
        assert (p.node_budget_per_seq, p.active_heads, p.topk_by_depth, p.actual_nodes) == (budget, heads, out_topk,
                                                                                              nodes)
    for f in d["fits"]:
        assert rp.fit_topk_to_budget(f["topk"], f["budget"], min_topk_by_depth=f["min"],
                                     depth_weight_decay=f["decay"]) == f["out"]
    for c in d["conf"]:
        assert rp.topk_from_confidence(c["conf"], c["base"], c["depth"], adaptive=True, min_topk_by_depth=c["min"],
                                       low=c["low"], high=c["high"]) == c["out"]


# ------------------------------------------------------------------ top-k
def test_topk_kept_set_matches_reference(golden_dir):
    # sample_from_logits' top_k branch (acceptance.py:68-79) on 48 seeded rows,
    # top_k in {1, 2, 7, 40, 96}, top_p in {1, 0.9, 0.5, 0.95}
    d = np.load(golden_dir / "topk.npz")
    compared = 0
    for r in range(d["logits"].shape[0]):
        V = int(d["vocab"][r])
        if d["margin"][r] < 1e-5:
            continue
        mine = native.kept_set(d["logits"][r, :V], float(d["temperature"][r]), float(d["top_p"][r]),
                               int(d["top_k"][r]))
        assert np.array_equal(mine, d["kept"][r, :V]), r
        compared += 1
    assert compared >= 40


def test_topk_sampler_matches_renormalised_kept_distribution():
    rng = np.random.default_rng(13)
    logits = (rng.standard_normal(300) * 2).astype(np.float32)
    order = np.argsort(-logits, kind="stable")
    for temp, top_k, top_p in ((1.0, 12, 1.0), (0.7, 30, 0.8)):
        p = np.exp((logits[order[:top_k]].astype(np.float64) - logits.max()) / temp)
        p /= p.sum()
        k = top_k - 1 if top_p >= 1.0 else int(np.argmax(np.cumsum(p) > top_p))
        want = np.zeros(300, dtype=bool)
        want[order[: k + 1]] = True
        assert np.array_equal(native.kept_set(logits, temp, top_p, top_k), want)
        q = np.zeros(300)
        q[order[: k + 1]] = p[: k + 1] / p[: k + 1].sum()
        u = native.philox_uniforms(22, np.arange(60_000), 3, 1)[:, 0]
        s = native.sample_rows(np.broadcast_to(logits, (60_000, 300)).copy(), u, temperature=temp, top_p=top_p,
                               top_k=top_k)
        assert want[s].all()
        freq = np.bincount(s, minlength=300) / s.size
        assert np.max(np.abs(freq - q)) < 0.015


def test_topk_edges():
    x = np.array([1.0, 2.0, 2.0, 2.0, 0.0, 2.0], dtype=np.float32)
    u = np.linspace(0, 1 - 2 ** -24, 64, dtype=np.float32)
    rows = np.broadcast_to(x, (64, 6)).copy()
    # ties go to the lower index: top_k = 2 keeps entries 1 and 2 of the four 2.0s
    assert native.kept_set(x, 1.0, 1.0, 2).tolist() == [False, True, True, False, False, False]
    assert set(native.sample_rows(rows, u, top_k=2).tolist()) == {1, 2}
    # top_k = 1 is the argmax for every u; top_k >= V (or <= 0) is no cut
    assert set(native.sample_rows(rows, u, top_k=1).tolist()) == {1}
    assert np.array_equal(native.sample_rows(rows, u, top_k=6), native.sample_rows(rows, u))
    assert np.array_equal(native.sample_rows(rows, u, top_k=0), native.sample_rows(rows, u))
    # with top_p the nucleus is taken over the k candidates' renormalised mass
    assert native.kept_set(x, 1.0, 0.3, 3).tolist() == [False, True, False, False, False, False]
    assert native.kept_set(x, 1.0, 0.5, 3).tolist() == [False, True, True, False, False, False]
    # greedy ignores top_k
    assert native.sample_rows(x, [0.9], do_sample=False, top_k=3)[0] == 1


# --------------------------------------------------------------- generate
GENERATE_RUNS = ["fixed_422", "conc_rep2", "adaptive", "nucleus_095", "chain_boot", "chain_noboot",
                 "chain_conc_p09", "topk_8", "topk_40_p09", "chain_topk16"]


def oracle_generate_run(r: dict):
    """The oracle's generate on config 1 for a fixture run description."""
    from flashgrpo_b200.utils import synthetic

    chain = r.get("proposal_mode", "medusa") == "chain"
    model = synthetic.build_model(1)
    st = synthetic.medusa_head_tensors(1, chain=chain)
    heads = [{"norm_w": st[f"heads.{i}.norm.weight"], "norm_b": st[f"heads.{i}.norm.bias"],
              "fc_w": st[f"heads.{i}.fc.weight"], "fc_b": st[f"heads.{i}.fc.bias"]} for i in range(3)]
    cell = {k[len("chain_cell."):]: v for k, v in st.items() if k.startswith("chain_cell.")} if chain else None
    ids, mask = synthetic.random_prompts(4, 128, 4096, seed=0)
    if r["repeats"] > 1:
        ids, mask = ids[:2], mask[:2]
    cfg = rp.OracleConfig(tree_mode=r["tree_mode"], cpeak_nodes=r.get("cpeak_nodes", 512),
                          max_tree_nodes_per_seq=r["max_tree_nodes_per_seq"], max_tree_depth=r["max_tree_depth"],
                          fixed_tree_topk_by_depth=tuple(r["fixed_tree_topk_by_depth"]),
                          top_p=r.get("top_p", 1.0), top_k=r.get("top_k"),
                          adaptive_tree_enabled=r.get("adaptive_tree_enabled", False),
                          adaptive_min_topk_by_depth=tuple(r.get("adaptive_min_topk_by_depth", (1, 1, 1))),
                          proposal_mode=r.get("proposal_mode", "medusa"), chain_cell=cell,
                          chain_bootstrap_from_medusa=r.get("chain_bootstrap_from_medusa", True))
    return rp.generate(model, heads, ids, mask, cfg, rp.CallOrderSampler(r["seed"]), repeats=r["repeats"],
                       max_length=128 + r["max_new"])


@pytest.mark.parametrize("name", GENERATE_RUNS)
def test_generate_matches_reference_config1(golden_dir, name):
    """The oracle's generate loop against the reference's own
    FlashMedusaDecoder.generate (stable top-k, fg-icdf-v1/v1n draws
    substituted), for MEDUSA and chain proposals, nucleus draws and adaptive
    widths: tokens and every deterministic statistic of the result dict."""
    d = json.loads((golden_dir / "generate_cfg1.json").read_text())[name]
    res = oracle_generate_run(d["run"])
    assert res["generated_token_ids"] == d["generated_token_ids"]
    for k in ("total_acc_length", "total_decoded_token_num", "total_verify_rounds", "total_correction_tokens",
              "total_accepted_medusa_tokens", "total_proposed_medusa_tokens"):
        assert res[k] == d[k], k
    assert math.isclose(res["average_accept_length"], d["average_accept_length"])
    compare_stats(res, d["stats"])

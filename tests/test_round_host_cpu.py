"""Host logic of the round on CPU: the internal-row bound of adaptive trees
and the compact row view that retires finished rows (no GPU, no kernels)."""
from __future__ import annotations

import itertools

import torch

from flashgrpo_b200.decoding.medusa_tree import TreePlan, dense_topology, internal_nodes, max_adaptive_internal


def _bfs_internal(widths, budget):
    """Independent count: BFS expansion of a dense tree up to `budget` nodes."""
    n, frontier, internal = 1, [0], set()
    for k in widths:
        nxt = []
        for p in frontier:
            for _ in range(k):
                if n >= budget:
                    break
                internal.add(p)
                nxt.append(n)
                n += 1
        frontier = nxt
        if not frontier or n >= budget:
            break
    return len(internal)


def test_adaptive_internal_bound_covers_every_adapted_tree():
    for base, budget in (([4, 3, 2], 16), ([4, 3, 2], 32), ([3, 2, 2], 10), ([5, 1], 8), ([2, 2, 2, 2], 64)):
        plan = TreePlan(budget, len(base), base, budget, "concurrency_aware")
        bound = max_adaptive_internal(plan)
        assert bound >= len(internal_nodes(dense_topology(plan)[0]))
        worst = 0
        for depth in range(1, len(base) + 1):
            for w in itertools.product(*[range(1, k + 1) for k in base[:depth]]):
                worst = max(worst, _bfs_internal(w, budget))
        assert bound == worst, (base, budget)
    # the case that needed it: narrower and deeper than the base plan
    plan = TreePlan(16, 3, [4, 3, 2], 16, "concurrency_aware")
    assert len(internal_nodes(dense_topology(plan)[0])) == 5 and max_adaptive_internal(plan) == 10


def test_round_view_gathers_and_scatters_only_its_rows(monkeypatch):
    from types import SimpleNamespace

    from flashgrpo_b200.engine import verify
    from flashgrpo_b200.engine.verify import DecodeState, ModelSpec, RoundView

    # the fg_kv_layer structs need device tensors: stand-ins that keep the row map
    monkeypatch.setattr(verify.ops, "kv_layer", lambda k, v, rows=None: SimpleNamespace(
        rows=None if rows is None else rows.data_ptr(), batch=0 if rows is None else k.shape[0]))

    spec = ModelSpec(n_layers=2, hidden=8, n_q_heads=2, n_kv_heads=1, head_dim=16, inter=16, vocab=32, eps=1e-6,
                     dtype=torch.float32)
    st = DecodeState(spec, 6, 20, torch.device("cpu"), n_heads=2)
    st.row_len.copy_(torch.tensor([10, 11, 12, 13, 14, 15], dtype=torch.int32))
    st.pending.copy_(torch.tensor([-1, 5, -1, 7, -1, 9], dtype=torch.int32))
    st.active.copy_(torch.tensor([1, 1, 0, 1, 1, 1], dtype=torch.int32))
    st.seq_ids.copy_(torch.arange(100, 106, dtype=torch.int32))
    st.hidden.copy_(torch.arange(48, dtype=torch.float32).view(6, 8))
    before = {k: getattr(st, k).clone() for k in ("row_len", "pending", "active", "seq_ids")}
    hidden0 = st.hidden.clone()
    v = RoundView(st, 3, n_heads=2)
    assert v.round_dev is st.round_dev and v.k is st.k
    assert all(kv.rows == v.rows.data_ptr() and kv.batch == 6 for kv in v.kv_layers)
    rows = [4, 1, 5]
    v.rows.copy_(torch.tensor(rows, dtype=torch.int32))
    v.gather()
    assert v.row_len.tolist() == [14, 11, 15] and v.pending.tolist() == [-1, 5, 9]
    assert v.seq_ids.tolist() == [104, 101, 105] and torch.equal(v.hidden, hidden0[rows])
    # a round advances the view's rows; scatter writes back exactly those rows
    v.row_len += 3
    v.pending.copy_(torch.tensor([2, -1, 4], dtype=torch.int32))
    v.active.copy_(torch.tensor([0, 1, 1], dtype=torch.int32))
    v.hidden.mul_(-1)
    v.scatter()
    assert st.row_len.tolist() == [10, 14, 12, 13, 17, 18]
    assert st.pending.tolist() == [-1, -1, -1, 7, 2, 4]
    assert st.active.tolist() == [1, 1, 0, 1, 0, 1]
    assert torch.equal(st.seq_ids, before["seq_ids"])
    for r in range(6):
        want = -hidden0[r] if r in rows else hidden0[r]
        assert torch.equal(st.hidden[r], want), r


def test_hf_plugin_registration_cache_and_ancestor_bits():
    from transformers import AttentionInterface

    from flashgrpo_b200.models.hf_tree_attention import FGStaticCache, ancestor_bits

    assert "fg_tree" in AttentionInterface._global_mapping
    cache = FGStaticCache.empty(2, 3, 2, 16, 8, dtype=torch.float32, device="cpu")
    cache.row_len.copy_(torch.tensor([0, 3, 5], dtype=torch.int32))
    k, v = torch.randn(3, 2, 4, 8), torch.randn(3, 2, 4, 8)
    cache.update(k, v, 1)
    for b, start in enumerate((0, 3, 5)):
        assert torch.equal(cache.k[1][b, :, start:start + 4], k[b]) and torch.equal(cache.v[1][b, :, start:start + 4],
                                                                                   v[b])
        assert torch.count_nonzero(cache.k[1][b, :, :start]) == 0
    assert torch.count_nonzero(cache.k[0]) == 0 and cache.row_len.tolist() == [0, 3, 5]
    # self + ancestors, as build_tree_attention_inputs; node 40 sits in word 1
    parents = [-1, 0, 0, 1, 2] + [4] * 36
    bits = ancestor_bits(parents)
    assert bits[:5, 0].tolist() == [0b1, 0b11, 0b101, 0b1011, 0b10101]
    assert bits[40].tolist()[0] == 0b10101 and bits[40].tolist()[1] == 1 << (40 - 32)


def test_new_entry_point_wrappers_check_their_buffers(monkeypatch):
    """The ops wrappers of fg_medusa_propose, fg_chain_step and
    fg_gate_up_silu hand the library well-sized outputs or raise: run on CPU
    tensors with the device checks and the library call stubbed out."""
    import pytest

    from flashgrpo_b200 import ops

    calls = []
    monkeypatch.setattr(ops, "_need", lambda *a, **k: None)
    monkeypatch.setattr(ops, "_stream", lambda t: 0)
    monkeypatch.setattr(ops.N, "call", lambda name, *a, **k: calls.append((name, k.get("n_launch"))))
    bf, i32, f32 = torch.bfloat16, torch.int32, torch.float32
    B, H, V, k = 4, 128, 300, 3
    heads = [dict(norm_w=torch.ones(H, dtype=bf), norm_b=torch.zeros(H, dtype=bf), fc_w=torch.zeros(H, H, dtype=bf),
                  fc_b=torch.zeros(H, dtype=bf)) for _ in range(2)]
    x = torch.zeros(3 * B, H, dtype=bf)
    w = torch.zeros(V, H, dtype=bf)
    top = lambda rows: (torch.zeros(rows, k, dtype=i32), torch.zeros(rows, k, dtype=f32), torch.zeros(rows, dtype=f32),
                        None)
    ws = torch.zeros(16, dtype=i32)
    ops.medusa_propose(x, B, heads, w, root_logits=torch.zeros(B, V, dtype=bf), k=k, topk_out=top(2 * B), workspace=ws)
    assert calls[-1] == ("fg_medusa_propose", 2 + 2 + 2)  # LayerNorm, 2 fc, finish, lm_head + merge
    with pytest.raises(ValueError):
        ops.medusa_propose(x, B, heads, w, root_logits=torch.zeros(B, V - 1, dtype=bf), k=k, topk_out=top(2 * B),
                           workspace=ws)
    with pytest.raises(ValueError):
        ops.medusa_propose(x, B, heads, w, root_logits=None, k=k, topk_out=top(2 * B - 1), workspace=ws)
    with pytest.raises(ValueError):
        ops.medusa_propose(x, B, heads, w, root_logits=None, k=k, topk_out=None, workspace=ws)
    # chain step: 2 sequences, 3 parents, fanout 2, 5 children each
    cell = {n: torch.zeros(2, dtype=bf) for n in ("state_norm.weight", "state_norm.bias", "token_norm.weight",
                                                  "token_norm.bias", "out_proj.bias", "gate")}
    cell.update({"state_proj.weight": torch.zeros(64, H, dtype=bf), "token_proj.weight": torch.zeros(64, H, dtype=bf),
                 "out_proj.weight": torch.zeros(H, 64, dtype=bf)})
    state = torch.zeros(6, H, dtype=bf)
    toks = torch.zeros(2, 6, dtype=i32)
    kw = dict(n_parent=3, fanout=2, n_child=5, embed=w, cell=cell, lm_head=w, k=k, workspace=ws)
    ops.chain_step(state, toks, state_out=torch.zeros(10, H, dtype=bf), topk_out=top(10), **kw)
    assert calls[-1] == ("fg_chain_step", 6 + 2)
    with pytest.raises(ValueError):
        ops.chain_step(state, toks, state_out=torch.zeros(9, H, dtype=bf), topk_out=top(10), **kw)
    with pytest.raises(ValueError):
        ops.chain_step(state, toks, state_out=torch.zeros(10, H, dtype=bf), topk_out=top(9), **kw)
    with pytest.raises(ValueError):
        ops.chain_step(state[:5], toks, state_out=torch.zeros(10, H, dtype=bf), topk_out=top(10), **kw)
    with pytest.raises(ValueError):
        ops.chain_step(state, toks, state_out=torch.zeros(10, H, dtype=bf), topk_out=top(10),
                       **{**kw, "embed": w[:V - 1]})
    # 9 heads: two LayerNorm and two finishing launches around the 9 fc GEMMs
    heads9 = heads * 4 + heads[:1]
    ops.medusa_propose(torch.zeros(10 * B, H, dtype=bf), B, heads9, w, root_logits=None, k=k, topk_out=top(9 * B),
                       workspace=ws)
    assert calls[-1] == ("fg_medusa_propose", 2 + 9 + 2 + 2)
    # 600 chain rows run as three 256-row passes
    ops.chain_step(torch.zeros(60 * 3, H, dtype=bf), torch.zeros(60, 10, dtype=i32), n_parent=3, fanout=4,
                   n_child=10, embed=w, cell=cell, lm_head=None, k=0, state_out=torch.zeros(600, H, dtype=bf),
                   topk_out=None, workspace=ws)
    assert calls[-1] == ("fg_chain_step", 3 * 6)
    # fused MLP
    xt, wgu = torch.zeros(7, H, dtype=bf), torch.zeros(2 * 256, H, dtype=bf)
    ops.gate_up_silu(xt, wgu, out=torch.zeros(7, 256, dtype=bf))
    assert calls[-1] == ("fg_gate_up_silu", None)
    with pytest.raises(ValueError):
        ops.gate_up_silu(xt, wgu, out=torch.zeros(7, 255, dtype=bf))


def test_round_tree_statistics_match_dense_topology():
    """The per-round tree counts the decoder derives from the device plan
    (widths, node count) equal those of the BFS tree itself: nodes per depth
    (CandidateTree.nodes_by_head) and the nodes that have children."""
    from flashgrpo_b200.decoding.flash_medusa_decoder import tree_internal_nodes, tree_level_counts

    for widths in ([4, 2], [4, 3, 2], [3, 2, 2], [8], [2, 2, 2, 2, 2], [1, 1, 1], [5, 4], [4, 1, 3]):
        for budget in range(1, 70):
            plan = TreePlan(budget, len(widths), list(widths), budget, "fixed")
            parents, depths = dense_topology(plan)
            n = len(parents)
            want_counts = [sum(1 for d in depths if d == dd) for dd in range(2, max(depths) + 1)]
            assert tree_level_counts(widths, n) == want_counts, (widths, budget)
            assert tree_internal_nodes(widths, n) == set(internal_nodes(parents)), (widths, budget)


def test_result_dict_covers_the_reference_keys(golden_dir):
    """generate()'s result carries every key the reference's result dict has
    (flash_medusa_decoder.py:3039-3117, recorded in the generate fixtures),
    assembled here from synthetic per-round outputs without a GPU."""
    import json

    from flashgrpo_b200.decoding.flash_medusa_decoder import RolloutStats

    ref_keys = set()
    for run in json.loads((golden_dir / "generate_cfg1.json").read_text()).values():
        ref_keys |= set(run["result_keys"])
    acc = RolloutStats(3)
    acc.round(4, 16, [4, 2], 13, [0, 1, 5, 0], True, 2, 0.01, [0.001, 0.006, 0.002])
    acc.rows([1, 2, 3, 1], [-1, 7, -1, -1])
    acc.round(4, 16, [4, 2], 13, [0, 0, 0, 0], True, 2, 0.01, None)
    acc.rows([1, 1, 1, 1], [-1, -1, 3, -1])
    res = acc.result([[1], [2, 3], [4, 5, 6], [7]], prefill_time=0.5, total_time=1.0, statistical_time=False,
                     cache_update_mode="extract_path")
    assert ref_keys - set(res) == set()
    assert res["tree_query_rows"] == 2 * 4 * 13
    # 5 internal nodes per tree; row 3's last node (5) is a leaf in round 1
    assert res["tree_lm_head_rows"] == 2 * 4 * 5 + 1
    assert res["tree_nodes_head1"] == 2 * 4 * 4 and res["tree_nodes_head2"] == 2 * 4 * 8
    assert res["tree_total_nodes"] == 2 * 4 * 12 + 8
    assert res["medusa_proposed_by_depth"] == {2: 32, 3: 64}
    assert res["accept_length_histogram"] == {1: 6, 2: 1, 3: 1}
    assert res["medusa_accept_by_depth"] == {2: 2, 3: 1}
    assert res["total_correction_tokens"] == 2 and res["timing_sample_count"] == 1
    assert res["actual_tree_layout_counts"] == {"configured": 8}
    # without statistical_time the wall time (0.02 s) is split by the sampled shares
    assert abs(res["tree_verify_time_cost"] - 0.02 * 6 / 9) < 1e-12
    assert abs(res["medusa_head_time_cost"] + res["tree_verify_time_cost"] + res["cache_update_time_cost"]
               - 0.02) < 1e-12


def test_bench_workloads_and_sweep_helpers():
    """bench.py's host side: the three GPU configurations' tree plans (config
    2: [4, 2] with 13 nodes; config 3: 4 heads, adaptive widths 2..8, 32
    nodes; config 4: chain proposals within 64 nodes), the config-5 trees
    (parents before children, depth <= 4 so accepted paths fit) and the
    single-point sweep option."""
    import sys
    from pathlib import Path

    import torch

    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    import bench

    c2 = bench.workload_config(2, 64, 1024, 28, 1)
    assert (c2["tree"], c2["tree_nodes"], c2["active_heads"]) == ([4, 2], 13, 2)
    c3 = bench.workload_config(3, 16, 2048, 28, 1)
    assert c3["tree_nodes"] == 32 and c3["medusa_heads"] == 4 and c3["adaptive_topk"] == [2, 8]
    c4 = bench.workload_config(4, 32, 4096, 32, 1)
    assert c4["proposal_mode"] == "chain" and c4["tree_nodes"] <= 64 and c4["layers"] == 32
    # the sharded global batch: every rank's config names its own rollouts
    assert bench.workload_config(2, 64, 1024, 28, 8)["parallelism"].startswith("dp8")
    g = torch.Generator().manual_seed(7)
    for n in (1, 8, 16, 64, 128):
        parents = bench.random_tree(n, g)
        assert parents[0] == -1 and all(0 <= parents[j] < j for j in range(1, n))
        depth = [0] * n
        for j in range(1, n):
            depth[j] = depth[parents[j]] + 1
        assert max(depth) <= 4
    old = sys.argv
    try:
        sys.argv = ["bench.py", "--sweep", "attention", "--sweep-only", "1024:8:32,16384:128:1"]
        args = bench.parse_args()
    finally:
        sys.argv = old
    assert args.sweep == "attention" and args.sweep_only == "1024:8:32,16384:128:1"
    assert (args.rows, args.prefix, args.e2e_prompt, args.e2e_len) == (64, 1024, 256, 1024)

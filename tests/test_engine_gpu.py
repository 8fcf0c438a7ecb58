"""End-to-end parity of the B200 verify engine and the drop-in decoder.

* config 1 (fp32): FlashMedusaDecoder.generate on the GPU against the oracle's
  restatement of the reference generate loop on the CPU, with the same
  per-(sequence, round, draw) Philox uniforms -> identical tokens and stats.
* a Qwen2.5-1.5B-shaped bf16 model with 2 layers: one verify round's tree
  hidden states against HF eager attention with the reference's dense mask
  (bf16 tolerance), and the acceptance outputs against the oracle walk fed the
  GPU's own tree logits (bit-exact).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import compare_stats, cuda_available
from oracle import native as orc
from oracle import reference_path as rp

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]


class _Tok:
    pad_token_id = 0
    eos_token_id = 1


def _heads_list(st, n):
    return [{"norm_w": st[f"heads.{i}.norm.weight"], "norm_b": st[f"heads.{i}.norm.bias"],
             "fc_w": st[f"heads.{i}.fc.weight"], "fc_b": st[f"heads.{i}.fc.bias"]} for i in range(n)]


@pytest.mark.parametrize("run", [
    dict(tree_mode="fixed", fixed=(4, 2, 2), mx=16, depth=4, repeats=1, max_new=24, seed=0),
    dict(tree_mode="concurrency_aware", cpeak=64, fixed=(4, 3, 2), mx=16, depth=4, repeats=2, max_new=16, seed=3),
    dict(tree_mode="concurrency_aware", cpeak=2048, fixed=(3, 2, 2), mx=32, depth=4, repeats=1, max_new=20, seed=9,
         greedy=True),
    # nucleus sampling, the reference's default top_p
    dict(tree_mode="fixed", fixed=(4, 2, 2), mx=16, depth=4, repeats=1, max_new=20, seed=5, top_p=0.95),
    # adaptive top-k from head confidences (two thresholds, quantile over the rows)
    dict(tree_mode="concurrency_aware", cpeak=128, fixed=(4, 3, 2), mx=32, depth=4, repeats=2, max_new=20, seed=7,
         adaptive=True),
    # chain proposals: per-parent top-k from the ChainDraftCell state, bootstrapped from head 1
    dict(tree_mode="fixed", fixed=(3, 2, 2), mx=16, depth=4, repeats=1, max_new=20, seed=13, chain=True),
    dict(tree_mode="fixed", fixed=(2, 2), mx=7, depth=3, repeats=2, max_new=16, seed=17, chain=True,
         bootstrap=False),
    # top-k draws, alone and with top_p
    dict(tree_mode="fixed", fixed=(4, 2, 2), mx=16, depth=4, repeats=1, max_new=20, seed=23, top_k=8),
    dict(tree_mode="concurrency_aware", cpeak=64, fixed=(4, 3, 2), mx=16, depth=4, repeats=2, max_new=16, seed=29,
         top_k=40, top_p=0.9),
    dict(tree_mode="fixed", fixed=(3, 2, 2), mx=16, depth=4, repeats=1, max_new=16, seed=31, chain=True, top_k=16),
])
def test_generate_config1_matches_oracle(run):
    from flashgrpo_b200.decoding.flash_medusa_decoder import FlashMedusaConfig, FlashMedusaDecoder
    from flashgrpo_b200.utils import synthetic

    cpu_model = synthetic.build_model(1)
    gpu_model = synthetic.build_model(1).cuda()
    chain = run.get("chain", False)
    st = synthetic.medusa_head_tensors(1, chain=chain)
    cell = {k[len("chain_cell."):]: v for k, v in st.items() if k.startswith("chain_cell.")} if chain else None
    ids, mask = synthetic.random_prompts(4, 128, 4096, seed=0)
    if run["repeats"] > 1:
        ids, mask = ids[:2], mask[:2]
    greedy = run.get("greedy", False)
    ocfg = rp.OracleConfig(tree_mode=run["tree_mode"], cpeak_nodes=run.get("cpeak", 512),
                           max_tree_nodes_per_seq=run["mx"], max_tree_depth=run["depth"],
                           fixed_tree_topk_by_depth=run["fixed"], do_sample=not greedy,
                           top_p=run.get("top_p", 1.0), top_k=run.get("top_k"),
                           adaptive_tree_enabled=run.get("adaptive", False),
                           adaptive_confidence_low=0.3, adaptive_confidence_high=0.9,
                           proposal_mode="chain" if chain else "medusa", chain_cell=cell,
                           chain_bootstrap_from_medusa=run.get("bootstrap", True))
    ref = rp.generate(cpu_model, _heads_list(st, 3), ids, mask, ocfg, rp.SeqRoundSampler(run["seed"]),
                      repeats=run["repeats"], max_length=128 + run["max_new"])
    cfg = FlashMedusaConfig(num_medusa_heads=3, tree_mode=run["tree_mode"], cpeak_nodes=run.get("cpeak", 512),
                            max_tree_nodes_per_seq=run["mx"], max_tree_depth=run["depth"],
                            fixed_tree_topk_by_depth=run["fixed"], top_p=run.get("top_p", 1.0),
                            top_k=run.get("top_k"), do_sample=not greedy,
                            adaptive_tree_enabled=run.get("adaptive", False), adaptive_confidence_low=0.3,
                            adaptive_confidence_high=0.9, proposal_mode="chain" if chain else "medusa",
                            chain_bootstrap_from_medusa=run.get("bootstrap", True),
                            sampling_seed=run["seed"])
    dec = FlashMedusaDecoder(gpu_model, {k: v.cuda() for k, v in st.items()}, _Tok(), cfg)
    res = dec.generate(ids, mask, repeated_generate_nums=run["repeats"], max_length=128 + run["max_new"])
    assert res["generated_token_ids"] == ref["generated_token_ids"]
    for k in ("total_acc_length", "total_decoded_token_num", "total_verify_rounds", "total_correction_tokens",
              "total_accepted_medusa_tokens", "total_proposed_medusa_tokens"):
        assert res[k] == ref[k], k
    # the rest of the reference's result statistics (tree rows, histograms, rates)
    want = {k: v for k, v in ref.items() if k not in ("generated_token_ids", "prefill_time", "round_times")}
    compare_stats(res, want)
    assert res["timing_sample_count"] >= 1 and res["sampled_tree_verify_cuda_time_s"] > 0
    assert res["kv_extraction_success_count"] == res["total_verify_rounds"]
    if run.get("adaptive"):
        # the confidences did shrink some trees below the base plan
        base = rp.plan_tree(active_batch_size=ids.shape[0] * run["repeats"], num_medusa_heads=3,
                            tree_mode=run["tree_mode"], cpeak_nodes=run.get("cpeak", 512), min_tree_nodes_per_seq=1,
                            max_tree_nodes_per_seq=run["mx"], max_tree_depth=run["depth"],
                            fixed_tree_topk_by_depth=list(run["fixed"]), adaptive_tree_enabled=True,
                            adaptive_min_topk_by_depth=[1, 1, 1])
        assert res["total_proposed_medusa_tokens"] < res["total_decoded_token_num"] * (base.actual_nodes - 1)
    from flashgrpo_b200 import _native

    assert _native.read_device_error(clear=True) == 0


@pytest.mark.parametrize("adaptive", [False, True])
def test_generate_retires_finished_rows(adaptive):
    """Rows that reach EOS at different rounds leave the batch (the reference's
    select_cache_batch); later rounds run on the remaining rows through a row
    map into the unmoved cache.  Tokens and statistics equal the oracle's,
    which drops finished rows by index_select -- with adaptive trees this also
    pins the confidence quantile to the active rows."""
    from flashgrpo_b200.decoding.flash_medusa_decoder import FlashMedusaConfig, FlashMedusaDecoder
    from flashgrpo_b200.utils import synthetic

    cpu_model = synthetic.build_model(1)
    gpu_model = synthetic.build_model(1).cuda()
    st = synthetic.medusa_head_tensors(1)
    ids, mask = synthetic.random_prompts(4, 128, 4096, seed=2)
    run = dict(tree_mode="concurrency_aware", cpeak_nodes=128, max_tree_nodes_per_seq=32, max_tree_depth=4,
               fixed_tree_topk_by_depth=(4, 3, 2), do_sample=True, top_p=1.0, adaptive_tree_enabled=adaptive,
               adaptive_confidence_low=0.3, adaptive_confidence_high=0.9)
    ocfg = rp.OracleConfig(**run)
    max_length = 128 + 24
    # an EOS token that one row emits early: that row retires while others go on
    free = rp.generate(cpu_model, _heads_list(st, 3), ids, mask, ocfg, rp.SeqRoundSampler(11), repeats=2,
                       max_length=max_length, eos_token_id=-1)
    eos = free["generated_token_ids"][0][3]
    ref = rp.generate(cpu_model, _heads_list(st, 3), ids, mask, ocfg, rp.SeqRoundSampler(11), repeats=2,
                      max_length=max_length, eos_token_id=eos)
    lens = [len(t) for t in ref["generated_token_ids"]]
    assert min(lens) < 24 and max(lens) > min(lens), lens  # rows retired at different rounds

    class Tok:
        pad_token_id = 0
        eos_token_id = eos

    cfg = FlashMedusaConfig(num_medusa_heads=3, sampling_seed=11, **run)
    dec = FlashMedusaDecoder(gpu_model, {k: v.cuda() for k, v in st.items()}, Tok(), cfg)
    for _ in range(2):  # the second call replays the graphs captured for the shrinking batches
        res = dec.generate(ids, mask, repeated_generate_nums=2, max_length=max_length)
        assert res["generated_token_ids"] == ref["generated_token_ids"]
        for k in ("total_acc_length", "total_decoded_token_num", "total_verify_rounds", "total_correction_tokens",
                  "total_accepted_medusa_tokens", "total_proposed_medusa_tokens"):
            assert res[k] == ref[k], k
        assert res["average_active_batch_size"] < 8
    from flashgrpo_b200 import _native

    assert _native.read_device_error(clear=True) == 0


@pytest.mark.parametrize("cfg_id,chain,topk,mx,cpeak", [
    (2, False, (4, 3, 2), 16, 128),
    (3, False, (4, 3, 2), 16, 128),
    # config 4: Llama layout, chain proposals, up to 64 nodes per sequence
    (4, True, (4, 4, 4), 64, 512),
])
def test_verify_round_bf16_against_hf_eager(cfg_id, chain, topk, mx, cpeak):
    """One round on configs 2-4's layer shapes (12/2 and 28/4 Qwen2 heads;
    32/8 Llama heads with RoPE theta 5e5), 2 layers each: tree hidden states
    and tree K/V against HF eager attention with the reference's dense mask,
    acceptance bit-exact against the oracle walk on the GPU's own logits,
    root draws, compaction and the next-round hidden state."""
    from flashgrpo_b200 import ops
    from flashgrpo_b200.decoding.medusa_tree import plan_tree
    from flashgrpo_b200.engine.verify import RoundConfig, VerifyEngine
    from flashgrpo_b200.utils import synthetic

    torch.manual_seed(0)
    model = synthetic.build_model(cfg_id, layers=2, device="cpu").cuda()
    st_heads = {k: v.cuda() for k, v in synthetic.medusa_head_tensors(cfg_id, chain=chain).items()}
    ids, mask = synthetic.random_prompts(2, 200, synthetic.CONFIGS[cfg_id]["vocab"], seed=4)
    eng = VerifyEngine(model, st_heads)
    plan_kw = dict(tree_mode="concurrency_aware", cpeak_nodes=cpeak, min_tree_nodes_per_seq=1,
                   max_tree_nodes_per_seq=mx, max_tree_depth=4, fixed_tree_topk_by_depth=list(topk))
    plan = plan_tree(active_batch_size=8, num_medusa_heads=3, **plan_kw)
    nh = plan.active_heads
    state = eng.prefill(ids, mask, repeats=4, capacity=200 + mx + 8, n_heads=nh)
    old_len = state.row_len.clone()
    k_before = state.k.clone()
    v_before = state.v.clone()
    rb = eng.buffers(8, plan, nh, nh + 2)
    n = rb.N
    if cfg_id == 2:
        assert (plan.topk_by_depth, n) == ([4, 2], 13)
    params = ops.plan_params(active_batch_size=8, num_medusa_heads=3, **plan_kw)
    cfg = RoundConfig(seed=5, chain=chain)
    with torch.inference_mode():
        hidden0 = state.hidden.clone()
        pending0 = state.pending.clone()
        if chain:
            eng.propose_chain(state, rb, cfg)
            eng.build_tree(state, rb, params)
            for off, cnt, tk in rb.chain_tokens:
                rb.tree["tokens"][:, off:off + cnt] = tk
        else:
            eng.propose(state, rb, cfg)
            eng.build_tree(state, rb, params)
        eng.verify_forward(state, rb, cfg)
        tree_hidden = rb.tree_hidden.clone()
        k_tree = state.k.clone()
        v_tree = state.v.clone()
        eng.accept(state, rb, cfg)
    torch.cuda.synchronize()
    assert int(rb.tree["plan"][10]) == n
    # --- tree hidden vs HF eager with the dense 4D mask over the prefill cache
    from transformers import DynamicCache

    tok = rb.tree["tokens"].long()
    pos = rb.tree["positions"].long()
    trees = [rp.Tree(tok[b].tolist(), rb.tree["parents"].tolist(), rb.tree["depths"].tolist()) for b in range(8)]
    L = int(old_len[0])
    full = torch.ones(8, L, dtype=torch.long, device="cuda")
    _, mask4d, _, _ = rp.tree_attention_inputs(trees, full.cpu(), old_len.cpu().long(), pad_token_id=0,
                                               dtype=torch.bfloat16)
    cache = DynamicCache()
    for l in range(2):
        cache.update(k_before[l, :, :, :L].clone(), v_before[l, :, :, :L].clone(), l)
    model.config._attn_implementation = "eager"
    with torch.inference_mode():
        ref = model.model(input_ids=tok, attention_mask=mask4d.cuda(), position_ids=pos, past_key_values=cache,
                          use_cache=True, return_dict=True).last_hidden_state
    # bf16 on both sides with different summation orders: 2e-2 relative in
    # norm, and no element further than 3e-2 of the largest magnitude
    d = tree_hidden.float() - ref.float()
    rel = (d.norm() / ref.float().norm()).item()
    err, scale = d.abs().max().item(), ref.float().abs().max().item()
    assert rel <= 2e-2 and err <= 3e-2 * scale, (rel, err, scale)
    # --- the tree K/V landed at each row's tail like DynamicCache.update appends them
    for l in range(2):
        ref_k = cache.layers[l].keys[:, :, L:L + n].float()
        dk = k_tree[l, :, :, L:L + n].float() - ref_k
        assert (dk.norm() / ref_k.norm()).item() <= 2e-2 and dk.abs().max() <= 3e-2 * ref_k.abs().max()
    # --- acceptance on the GPU's own tree logits equals the oracle walk
    U = rb.U.cpu().numpy()
    walk = orc.accept_walk(rb.tree_logits.float().cpu().numpy(), rb.tree["slot"].cpu().numpy(),
                           rb.tree["tokens"].cpu().numpy(),
                           np.tile(rb.tree["parents"].cpu().numpy(), (8, 1)), np.full(8, n), U[:, 1:].copy(),
                           do_sample=True, temperature=1.0, eos_id=1, max_length=1 << 30,
                           row_len=old_len.cpu().numpy(), dcap=nh + 2)
    for k in ("acc_tokens", "acc_nodes", "acc_len", "correction", "last_node", "finished"):
        assert np.array_equal(rb.out[k].cpu().numpy(), walk[k]), k
    assert np.array_equal(state.pending.cpu().numpy(), walk["pending"])
    assert torch.equal(state.row_len.cpu(), old_len.cpu() + torch.from_numpy(walk["acc_len"]))
    # root tokens: fg-icdf-v1 draws on the GPU's root logits with the same uniforms
    root_ref = orc.sample_rows(rb.logits[:8].float().cpu().numpy(), U[:, 0].copy())
    root_ref = np.where(pending0.cpu().numpy() >= 0, pending0.cpu().numpy(), root_ref)
    assert np.array_equal(rb.root.cpu().numpy(), root_ref)
    # KV compaction: valid slots hold the accepted path's tree K/V
    for b in range(8):
        a = int(walk["acc_len"][b])
        for j in range(a):
            src = L + int(walk["acc_nodes"][b, j])
            assert torch.equal(state.k[:, b, :, L + j], k_tree[:, b, :, src])
            assert torch.equal(state.v[:, b, :, L + j], v_tree[:, b, :, src])
        assert torch.equal(state.hidden[b], tree_hidden[b, int(walk["last_node"][b])])
    assert not torch.equal(state.hidden, hidden0)


@pytest.mark.parametrize("cfg_id", [2, 4])
def test_hf_attention_plugin_matches_eager(cfg_id):
    """attn_implementation="fg_tree" inside the HF decoder (FGStaticCache +
    ancestor bits, no dense mask) gives the hidden states of HF eager
    attention with the reference's dense tree mask over a DynamicCache, and
    the cache holds the tree K/V at each row's tail with lengths unchanged."""
    from transformers import DynamicCache

    from flashgrpo_b200.models.hf_tree_attention import FGStaticCache, TreeInputs, ancestor_bits
    from flashgrpo_b200.utils import synthetic

    torch.manual_seed(0)
    model = synthetic.build_model(cfg_id, layers=2, device="cpu").cuda()
    spec = synthetic.CONFIGS[cfg_id]
    B, P = 4, 150
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, spec["vocab"], (B, P), generator=g).cuda()
    model.config._attn_implementation = "eager"
    with torch.inference_mode():
        pre = model.model(input_ids=prompt, use_cache=True, return_dict=True).past_key_values
    parents = [-1, 0, 0, 0, 0, 1, 1, 2, 2, 3, 3, 4, 4]
    depths = [1] + [0] * (len(parents) - 1)
    for i in range(1, len(parents)):
        depths[i] = depths[parents[i]] + 1
    n = len(parents)
    tokens = torch.randint(0, spec["vocab"], (B, n), generator=g).cuda()
    pos = (P + torch.tensor(depths) - 1).repeat(B, 1).cuda()
    # reference: eager attention, dense mask, DynamicCache appending the tree
    trees = [rp.Tree(tokens[b].tolist(), parents, depths) for b in range(B)]
    _, mask4d, _, _ = rp.tree_attention_inputs(trees, torch.ones(B, P, dtype=torch.long),
                                               torch.full((B,), P, dtype=torch.long), pad_token_id=0,
                                               dtype=spec["dtype"])
    dyn = DynamicCache()
    for l in range(2):
        dyn.update(pre.layers[l].keys.clone(), pre.layers[l].values.clone(), l)
    with torch.inference_mode():
        ref = model.model(input_ids=tokens, attention_mask=mask4d.cuda(), position_ids=pos, past_key_values=dyn,
                          use_cache=True, return_dict=True).last_hidden_state
    # the plugin
    cache = FGStaticCache.empty(2, B, spec["kv_heads"], P + n + 8, spec["head_dim"], dtype=spec["dtype"],
                                device="cuda")
    for l in range(2):
        cache.k[l][:, :, :P] = pre.layers[l].keys
        cache.v[l][:, :, :P] = pre.layers[l].values
    cache.row_len.fill_(P)
    model.config._attn_implementation = "fg_tree"
    try:
        with torch.inference_mode():
            out = model.model(input_ids=tokens, position_ids=pos, past_key_values=cache, use_cache=True,
                              return_dict=True, fg_tree=TreeInputs(cache, ancestor_bits(parents, "cuda")))
    finally:
        model.config._attn_implementation = "eager"
    d = out.last_hidden_state.float() - ref.float()
    rel = (d.norm() / ref.float().norm()).item()
    assert rel <= 2e-2 and d.abs().max().item() <= 3e-2 * ref.float().abs().max().item(), rel
    assert torch.equal(cache.row_len, torch.full_like(cache.row_len, P))
    for l in range(2):
        want = dyn.layers[l].keys[:, :, P:P + n].float()
        got = cache.k[l][:, :, P:P + n].float()
        assert ((got - want).norm() / want.norm()).item() <= 2e-2
    from flashgrpo_b200 import _native

    assert _native.read_device_error(clear=True) == 0


def test_extracted_cache_matches_recompute():
    # scripts/test_kv_extraction.py:29-85: after a verify round, the cache the
    # extract_path compaction leaves behind must be the cache a plain forward
    # over prompt + accepted tokens builds, and the next-round hidden state
    # must be that forward's last hidden state.
    from flashgrpo_b200 import ops
    from flashgrpo_b200.decoding.medusa_tree import plan_tree
    from flashgrpo_b200.engine.verify import RoundConfig, VerifyEngine
    from flashgrpo_b200.utils import synthetic

    torch.manual_seed(0)
    model = synthetic.build_model(1).cuda()
    heads = {k: v.cuda() for k, v in synthetic.medusa_head_tensors(1).items()}
    ids, mask = synthetic.random_prompts(4, 40, 4096, seed=21)
    eng = VerifyEngine(model, heads)
    plan = plan_tree(active_batch_size=4, num_medusa_heads=3, tree_mode="fixed", cpeak_nodes=512,
                     min_tree_nodes_per_seq=1, max_tree_nodes_per_seq=16, max_tree_depth=4,
                     fixed_tree_topk_by_depth=[4, 2, 2])
    params = ops.plan_params(tree_mode="fixed", active_batch_size=4, num_medusa_heads=3, cpeak_nodes=512,
                             min_tree_nodes_per_seq=1, max_tree_nodes_per_seq=16, max_tree_depth=4,
                             fixed_tree_topk_by_depth=(4, 2, 2))
    st = eng.prefill(ids, mask, repeats=1, capacity=80, n_heads=plan.active_heads)
    rb = eng.buffers(4, plan, plan.active_heads, plan.active_heads + 2)
    cfg = RoundConfig(do_sample=False, seed=3)  # greedy: long accepted paths on the peaked heads
    with torch.inference_mode():
        old_len = st.row_len.clone()
        eng.run_round(st, rb, params, cfg)
        eng.run_round(st, rb, params, cfg)  # a second round extracts on top of the first
    torch.cuda.synchronize()
    n_new = (st.row_len - old_len).tolist()
    assert max(n_new) >= 3
    model.config._attn_implementation = "eager"
    # the same two rounds on a fresh state, recording each round's accepted tokens
    st2 = eng.prefill(ids, mask, repeats=1, capacity=80, n_heads=plan.active_heads)
    with torch.inference_mode():
        rounds = []
        for _ in range(2):
            eng.run_round(st2, rb, params, cfg)
            a = rb.out["acc_len"].tolist()
            t = rb.out["acc_tokens"].tolist()
            rounds.append([t[b][: a[b]] for b in range(4)])
    torch.cuda.synchronize()
    assert (st2.row_len - old_len).tolist() == n_new  # the state object is reused: same rounds, same lengths
    L = int(old_len[0])
    for b in range(4):
        acc = rounds[0][b] + rounds[1][b]
        assert len(acc) == n_new[b]
        full = torch.cat([ids[b].cuda(), torch.tensor(acc, device="cuda")])[None]
        with torch.inference_mode():
            out = model.model(input_ids=full, use_cache=True, return_dict=True)
        ref_h = out.last_hidden_state[0, -1]
        # the engine's next-round hidden is the final-norm hidden of the last accepted node
        assert torch.allclose(st2.hidden[b], ref_h, atol=5e-3, rtol=5e-3), b
        for l, layer in enumerate(out.past_key_values.layers):
            n = L + len(acc)
            assert torch.allclose(st2.k[l, b, :, :n], layer.keys[0, :, :n], atol=5e-3, rtol=5e-3), (b, l)
            assert torch.allclose(st2.v[l, b, :, :n], layer.values[0, :, :n], atol=5e-3, rtol=5e-3), (b, l)

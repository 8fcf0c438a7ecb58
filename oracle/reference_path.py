"""Python restatement of the reference's MEDUSA tree-verify path (CPU, fp32).

TEST INFRASTRUCTURE ONLY.  This module is the checker for the product
package; the product never imports it.  It restates, in its own code, the
behaviour of these reference functions (paths inside ihbkaiser/ss-GRPO):

* ``dense_node_count``      flashgrpo_b200/decoding/medusa_tree.py:286-292
* ``fit_topk_to_budget``    flashgrpo_b200/decoding/medusa_tree.py:295-339
* ``plan_tree`` (dense)     flashgrpo_b200/decoding/medusa_tree.py:342-459
* ``build_batch_trees``     flashgrpo_b200/decoding/medusa_tree.py:758-799
* ``tree_attention_inputs`` flashgrpo_b200/decoding/tree_attention.py:6-67
* adaptive top-k            flashgrpo_b200/decoding/flash_medusa_decoder.py:1021-1095
* packed internal logits    flashgrpo_b200/decoding/flash_medusa_decoder.py:1097-1139
* acceptance walk           flashgrpo_b200/decoding/acceptance.py:183-267
* post-accept bookkeeping   flashgrpo_b200/decoding/flash_medusa_decoder.py:2289-2343
* extract_path              flashgrpo_b200/decoding/kv_extraction.py:34-218
* generate loop (no Reflex) flashgrpo_b200/decoding/flash_medusa_decoder.py:1272-3117
* model wrapper             flashgrpo_b200/models/qwen_flashgrpo_wrapper.py:100-239

Top-k uses the explicit tie rule (value descending, index ascending) instead
of ``torch.topk``, whose tie order is unspecified.  Sampling goes through a
pluggable ``Sampler`` so the same walk can run with the reference-pinning
uniform stream (``CallOrderSampler``) or with the product's per
(sequence, round, draw) Philox uniforms (``SeqRoundSampler``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from oracle import native

# ----------------------------------------------------------------- planner


def dense_node_count(topk_by_depth) -> int:
    total, width = 1, 1
    for k in topk_by_depth:
        width *= int(k)
        total += width
    return total


def fit_topk_to_budget(topk_by_depth, node_budget, *, min_topk_by_depth=None, depth_weight_decay=0.5):
    budget = max(1, int(node_budget))
    fitted = [max(1, int(k)) for k in topk_by_depth]
    raw_min = list(min_topk_by_depth or [])
    floor_k = [max(1, min(fitted[d], int(raw_min[d]) if d < len(raw_min) else 1)) for d in range(len(fitted))]
    while fitted and dense_node_count(fitted) > budget:
        best = None
        for d, value in enumerate(fitted):
            if value <= floor_k[d]:
                continue
            trial = fitted[:d] + [value - 1] + fitted[d + 1:]
            saved = dense_node_count(fitted) - dense_node_count(trial)
            loss = max(float(depth_weight_decay), 1e-3) ** d * (math.log1p(value) - math.log(value))
            key = (saved / max(loss, 1e-9), saved, d)
            if best is None or key > best:
                best = key
        if best is not None:
            fitted[best[2]] -= 1
        else:
            fitted.pop()
            floor_k.pop()
    return fitted


@dataclass
class Plan:
    node_budget_per_seq: int
    active_heads: int
    topk_by_depth: list
    actual_nodes: int
    mode: str
    layout: str = "dense"


def plan_tree(*, active_batch_size, num_medusa_heads, tree_mode, cpeak_nodes, min_tree_nodes_per_seq,
              max_tree_nodes_per_seq, max_tree_depth, fixed_tree_topk_by_depth, adaptive_tree_enabled=False,
              adaptive_min_topk_by_depth=None, tree_layout="dense") -> Plan:
    if tree_layout != "dense":
        raise ValueError("only the dense tree layout is restated")
    bsz = max(1, int(active_batch_size))
    if tree_mode == "fixed":
        budget = int(max_tree_nodes_per_seq)
        topk = [max(1, int(k)) for k in list(fixed_tree_topk_by_depth)[:num_medusa_heads]]
        while topk and dense_node_count(topk) > budget:
            topk[-1] -= 1
            if topk[-1] <= 0:
                topk.pop()
        heads = min(len(topk), max(0, int(max_tree_depth) - 1))
        topk = topk[:heads]
    elif tree_mode == "concurrency_aware":
        budget = max(int(min_tree_nodes_per_seq), min(int(max_tree_nodes_per_seq), int(cpeak_nodes) // bsz))
        max_heads = min(int(num_medusa_heads), max(0, int(max_tree_depth) - 1))
        defaults = list(fixed_tree_topk_by_depth) or [4, 3, 2, 1, 1]
        topk = []
        if adaptive_tree_enabled:
            raw_min = list(adaptive_min_topk_by_depth or [])
            minimum = []
            for d in range(max_heads):
                mk = max(1, int(raw_min[d]) if d < len(raw_min) else 1)
                if dense_node_count(minimum + [mk]) > budget:
                    break
                minimum.append(mk)
                topk.append(max(mk, int(defaults[min(d, len(defaults) - 1)])))
        else:
            width, used = 1, 1
            for d in range(max_heads):
                want = int(defaults[min(d, len(defaults) - 1)])
                room = budget - used
                if room <= 0:
                    break
                k = min(max(1, want), max(1, room // width))
                if used + width * k > budget:
                    k = room // width
                if k <= 0:
                    break
                topk.append(int(k))
                width *= int(k)
                used += width
    else:
        raise ValueError(f"Unsupported tree_mode={tree_mode}")
    return Plan(budget, len(topk), topk, dense_node_count(topk), tree_mode)


# ------------------------------------------------------------------- trees


@dataclass
class Tree:
    tokens: list
    parents: list
    depths: list

    def __post_init__(self):
        self.children = {}
        for i, p in enumerate(self.parents):
            if p >= 0:
                self.children.setdefault(p, []).append(i)

    @property
    def node_count(self):
        return len(self.tokens)

    def ancestors_including_self(self, i):
        chain = [i]
        while self.parents[chain[-1]] >= 0:
            chain.append(self.parents[chain[-1]])
        return chain[::-1]


def stable_topk(logits: torch.Tensor, k: int):
    """Top-k with ties broken by the lower vocabulary index."""
    values, idx = torch.sort(logits.float(), dim=-1, descending=True, stable=True)
    return values[..., :k], idx[..., :k]


def build_dense_trees(root_tokens, head_logits, plan: Plan) -> list[Tree]:
    B = len(root_tokens)
    cands = []
    for d, k in enumerate(plan.topk_by_depth[: plan.active_heads]):
        if d >= len(head_logits):
            break
        k = min(max(0, int(k)), int(head_logits[d].shape[-1]))
        if k <= 0:
            break
        cands.append(stable_topk(head_logits[d], k)[1].tolist())
    trees = []
    for b in range(B):
        tokens, parents, depths = [int(root_tokens[b])], [-1], [1]
        frontier = [0]
        for d, rows in enumerate(cands):
            nxt = []
            full = False
            for p in frontier:
                for tok in rows[b]:
                    tokens.append(int(tok))
                    parents.append(p)
                    depths.append(d + 2)
                    nxt.append(len(tokens) - 1)
                    if len(tokens) >= plan.node_budget_per_seq:
                        full = True
                        break
                if full:
                    break
            frontier = nxt
            if not frontier or len(tokens) >= plan.node_budget_per_seq:
                break
        trees.append(Tree(tokens, parents, depths))
    return trees


def chain_cell_forward(cell, state, token_embedding):
    """ChainDraftCell.forward (medusa_heads.py:154-160):
    state + sigmoid(gate) * out_proj(SiLU(state_proj(LN(state)) + token_proj(LN(embedding))))."""
    F = torch.nn.functional
    dt = cell["state_norm.weight"].dtype
    s = state.to(dt)
    t = token_embedding.to(dt)
    H = s.shape[-1]
    mixed = (F.linear(F.layer_norm(s, (H,), cell["state_norm.weight"], cell["state_norm.bias"], 1e-5),
                      cell["state_proj.weight"])
             + F.linear(F.layer_norm(t, (H,), cell["token_norm.weight"], cell["token_norm.bias"], 1e-5),
                        cell["token_proj.weight"]))
    delta = F.linear(F.silu(mixed), cell["out_proj.weight"], cell["out_proj.bias"])
    return s + torch.sigmoid(cell["gate"]) * delta


def build_chain_trees(root_tokens, cur_hidden, plan: Plan, heads, cell, lm_w, embed_w, *,
                      bootstrap_from_medusa=True) -> list[Tree]:
    """_build_chain_batch_trees (flash_medusa_decoder.py:1141-1261) with Reflex
    off and fixed widths: per depth, the lm_head of every parent state, its
    top-k (stable ties), children in parent then rank order under the node
    budget, and the next states from the chain cell on the chosen tokens."""
    B = len(root_tokens)
    tokens = [[int(t)] for t in root_tokens]
    parents = [[-1] for _ in range(B)]
    depths = [[1] for _ in range(B)]
    root = torch.as_tensor([int(t) for t in root_tokens], dtype=torch.long)
    if bootstrap_from_medusa and heads:
        states = project_heads(heads, cur_hidden, 1)[0]
    else:
        states = chain_cell_forward(cell, cur_hidden, embed_w[root])
    parent_rows = list(range(B))
    parent_nodes = [0] * B
    budget = plan.node_budget_per_seq
    for d, k in enumerate(plan.topk_by_depth):
        if states.shape[0] == 0:
            break
        logits = torch.nan_to_num(torch.nn.functional.linear(states.to(lm_w.dtype), lm_w).float(), nan=-1.0e9,
                                  posinf=1.0e9, neginf=-1.0e9)
        idx = stable_topk(logits, min(int(k), logits.shape[-1]))[1].tolist()
        nxt_state, nxt_tok, nxt_rows, nxt_nodes = [], [], [], []
        for ps, row in enumerate(parent_rows):
            if len(tokens[row]) >= budget:
                continue
            for tok in idx[ps]:
                if len(tokens[row]) >= budget:
                    break
                tokens[row].append(int(tok))
                parents[row].append(parent_nodes[ps])
                depths[row].append(d + 2)
                nxt_state.append(ps)
                nxt_tok.append(int(tok))
                nxt_rows.append(row)
                nxt_nodes.append(len(tokens[row]) - 1)
        if not nxt_tok:
            break
        states = chain_cell_forward(cell, states[torch.as_tensor(nxt_state)], embed_w[torch.as_tensor(nxt_tok)])
        parent_rows, parent_nodes = nxt_rows, nxt_nodes
    return [Tree(tokens[b], parents[b], depths[b]) for b in range(B)]


def tree_attention_inputs(trees, full_attention_mask, logical_lengths, *, pad_token_id, dtype):
    """Dense ancestor-only mask, positions logical_len + depth - 1, padding."""
    B = len(trees)
    nmax = max(max(t.node_count, 1) for t in trees)
    past = full_attention_mask.shape[1]
    ids = torch.full((B, nmax), int(pad_token_id), dtype=torch.long)
    depth = torch.ones((B, nmax), dtype=torch.long)
    valid = torch.zeros((B, nmax), dtype=torch.bool)
    allowed_tree = torch.zeros((B, nmax, nmax), dtype=torch.bool)
    for b, t in enumerate(trees):
        n = t.node_count
        ids[b, :n] = torch.tensor(t.tokens)
        depth[b, :n] = torch.tensor(t.depths)
        valid[b, :n] = True
        for i in range(n):
            for a in t.ancestors_including_self(i):
                allowed_tree[b, i, a] = True
        for i in range(n, nmax):
            allowed_tree[b, i, i] = True
    pos = logical_lengths.long().unsqueeze(1) + depth - 1
    pos = pos.masked_fill(~valid, 0)
    allowed = torch.cat(
        [full_attention_mask.bool()[:, None, :].expand(B, nmax, past), allowed_tree], dim=-1
    ).unsqueeze(1)
    mask = torch.zeros((B, 1, nmax, past + nmax), dtype=dtype).masked_fill(~allowed, torch.finfo(dtype).min)
    return ids, mask, pos, valid


def internal_logit_layout(trees):
    """Packed lm_head rows for nodes that have children, row-major (row, node)."""
    nmax = max((t.node_count for t in trees), default=1)
    rows, nodes = [], []
    slots = [[-1] * nmax for _ in trees]
    for b, t in enumerate(trees):
        for i in range(t.node_count):
            if t.children.get(i):
                slots[b][i] = len(rows)
                rows.append(b)
                nodes.append(i)
    return rows, nodes, slots


# ---------------------------------------------------------------- adaptive


def confidences(head_logits, metric="top1_prob", quantile=0.25):
    scores = []
    for lg in head_logits:
        if metric == "margin":
            # values only (tie order is irrelevant), subtracted in the logits dtype
            v = torch.topk(lg, k=min(2, lg.shape[-1]), dim=-1).values
            s = v[..., 0] if v.shape[-1] == 1 else v[..., 0] - v[..., 1]
        else:
            top1 = lg.max(dim=-1).values.float()
            s = torch.exp(top1 - torch.logsumexp(lg, dim=-1).float())
        scores.append(torch.nan_to_num(s.float(), nan=0.0, posinf=0.0, neginf=0.0))
    q = min(1.0, max(0.0, float(quantile)))
    return torch.quantile(torch.stack(scores), q, dim=-1).tolist()


def topk_from_confidence(conf, base_k, depth_idx, *, adaptive, min_topk_by_depth, low, high):
    base_k = max(1, int(base_k))
    mins = list(min_topk_by_depth) or [1]
    min_k = max(1, min(base_k, int(mins[min(depth_idx, len(mins) - 1)])))
    if not adaptive or base_k <= min_k:
        return base_k
    if not math.isfinite(float(conf)):
        return min_k
    if high <= low:
        return min_k if conf >= high else base_k
    if conf <= low:
        return base_k
    if conf >= high:
        return min_k
    ratio = (conf - low) / (high - low)
    return max(min_k, min(base_k, int(round(base_k - ratio * (base_k - min_k)))))


# ----------------------------------------------------------------- sampler


class CallOrderSampler:
    """Uniform for row k of the c-th sampler call = Philox(seed, (k, c, 0, 0))."""

    def __init__(self, seed=0):
        self.seed = int(seed)
        self.calls = 0

    def __call__(self, logits_rows: torch.Tensor, seq_ids, round_idx, draw, *, do_sample, temperature, top_p=1.0,
                 top_k=None):
        u = np.array([native.uniform(self.seed, k, self.calls, 0) for k in range(logits_rows.shape[0])],
                     dtype=np.float32)
        self.calls += 1
        return native.sample_rows(logits_rows.float().numpy(), u, do_sample=do_sample, temperature=temperature,
                                  top_p=top_p, top_k=top_k)


class SeqRoundSampler:
    """Uniform for (sequence id, verify round, draw) = Philox(seed, (seq, round, draw, 0)).

    Draw 0 is the root sample of the round; draw 1 + d is acceptance step d.
    """

    def __init__(self, seed=0):
        self.seed = int(seed)

    def __call__(self, logits_rows, seq_ids, round_idx, draw, *, do_sample, temperature, top_p=1.0, top_k=None):
        u = np.array([native.uniform(self.seed, int(s), int(round_idx), int(draw)) for s in seq_ids], dtype=np.float32)
        return native.sample_rows(logits_rows.float().numpy(), u, do_sample=do_sample, temperature=temperature,
                                  top_p=top_p, top_k=top_k)


def _cut_kwargs(top_p, top_k) -> dict:
    """top_p / top_k keyword arguments, passed only when they cut anything."""
    kw = {}
    if top_p is not None and top_p != 1.0:
        kw["top_p"] = top_p
    if top_k is not None:
        kw["top_k"] = int(top_k)
    return kw


def accept_walk_batch(trees, tree_logits, slots, sampler, seq_ids, round_idx, *, do_sample, temperature, top_p=1.0,
                      top_k=None):
    """Depth-synchronous exact_target walk (acceptance.py:183-267)."""
    B = len(trees)
    acc_tokens = [[int(t.tokens[0])] for t in trees]
    acc_nodes = [[0] for _ in trees]
    parent = [0] * B
    correction = [None] * B
    active = [b for b, t in enumerate(trees) if t.children.get(0)]
    step = 0
    while active:
        rows = torch.stack([tree_logits[slots[b][parent[b]]] for b in active])
        sampled = sampler(rows, [seq_ids[b] for b in active], round_idx, 1 + step,
                          do_sample=do_sample, temperature=temperature, **_cut_kwargs(top_p, top_k))
        step += 1
        still = []
        for b, tok in zip(active, sampled.tolist()):
            t = trees[b]
            hit = next((c for c in t.children.get(parent[b], []) if int(t.tokens[c]) == int(tok)), None)
            if hit is None:
                correction[b] = int(tok)
                continue
            acc_tokens[b].append(int(tok))
            acc_nodes[b].append(int(hit))
            parent[b] = int(hit)
            if t.children.get(int(hit)):
                still.append(b)
        active = still
    return acc_tokens, acc_nodes, parent, correction


# ------------------------------------------------------------ model helpers


def _cache_layers(cache):
    return [(layer.keys, layer.values) for layer in cache.layers]


def _new_cache(model):
    from transformers import DynamicCache

    try:
        return DynamicCache(config=model.config)
    except TypeError:
        return DynamicCache()


def _cache_from_layers(model, layers):
    cache = _new_cache(model)
    for i, (k, v) in enumerate(layers):
        cache.update(k, v, i)
    return cache


def _run_model(model, ids, mask, pos, cache):
    out = model.model(input_ids=ids, attention_mask=mask, position_ids=pos, past_key_values=cache, use_cache=True,
                      return_dict=True)
    return out.last_hidden_state, out.past_key_values


def extract_path_hf(cache_layers, old_len, accepted_nodes):
    """kv_extraction.py:34-84 on [B, H, S, D] tensors: pad by repeating the last node."""
    max_len = max(len(p) for p in accepted_nodes)
    idx = torch.tensor([[old_len + int(n) for n in (list(p) + [p[-1]] * (max_len - len(p)))] for p in accepted_nodes],
                       dtype=torch.long)
    out = []
    for k, v in cache_layers:
        new = []
        for t in (k, v):
            B, H, _, D = t.shape
            gathered = t.gather(2, idx[:, None, :, None].expand(B, H, max_len, D)).contiguous()
            t[:, :, old_len:old_len + max_len].copy_(gathered)
            new.append(t[:, :, :old_len + max_len])
        out.append(tuple(new))
    return out, max_len


# ------------------------------------------------------------ generate loop


@dataclass
class OracleConfig:
    num_medusa_heads: int = 3
    tree_mode: str = "concurrency_aware"
    cpeak_nodes: int = 512
    min_tree_nodes_per_seq: int = 1
    max_tree_nodes_per_seq: int = 10
    max_tree_depth: int = 4
    fixed_tree_topk_by_depth: tuple = (4, 3, 2)
    do_sample: bool = True
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int | None = None
    adaptive_tree_enabled: bool = False
    adaptive_confidence_metric: str = "top1_prob"
    adaptive_confidence_quantile: float = 0.25
    adaptive_confidence_low: float = 0.15
    adaptive_confidence_high: float = 0.45
    adaptive_min_topk_by_depth: tuple = (1, 1, 1)
    adaptive_depth_weight_decay: float = 0.5
    project_internal_tree_logits_only: bool = True
    proposal_mode: str = "medusa"          # "chain": ChainDraftCell proposals
    chain_bootstrap_from_medusa: bool = True
    chain_cell: dict | None = None         # chain_cell.* tensors keyed without the prefix


@dataclass
class RoundRecord:
    trees: list
    plan: Plan
    accepted: list
    accepted_nodes: list
    corrections: list
    pending: dict
    finished: list
    active_seq_ids: list
    old_lens: list
    extra: dict = field(default_factory=dict)


def project_heads(heads, hidden, n_heads):
    """MedusaPredictionHead.project_hidden for the first n_heads heads (medusa_heads.py:240-244)."""
    out = []
    for i in range(n_heads):
        h = heads[i]
        x = hidden.to(h["norm_w"].dtype)
        y = torch.nn.functional.layer_norm(x, (x.shape[-1],), h["norm_w"], h["norm_b"], 1e-5)
        y = torch.nn.functional.silu(torch.nn.functional.linear(y, h["fc_w"], h["fc_b"]))
        out.append(x + y)
    return out


@torch.no_grad()
def generate(model, heads, input_ids, attention_mask, cfg: OracleConfig, sampler, *, repeats=1, max_length=2048,
             pad_token_id=0, eos_token_id=1, record=None, prefill_fn=None):
    """Restatement of FlashMedusaDecoder.generate (Reflex off, MEDUSA proposal,
    exact_target acceptance, extract_path cache update, CPU fp32).

    ``heads`` is a list of dicts with norm_w, norm_b, fc_w, fc_b tensors.
    ``record`` (a list) receives one RoundRecord per verify round.
    ``prefill_fn(model, input_ids, attention_mask, pos, cache) -> (hidden,
    cache)`` replaces the model's prefill forward (host timing runs that only
    need the prefix's shape use it to skip a long CPU prefill).
    """
    import time

    t_start = time.perf_counter()
    round_times = []
    lm_w = model.lm_head.weight
    # prefill (wrapper.py:189-199): positions from the mask, fresh cache
    pos = (attention_mask.long().cumsum(-1) - 1).masked_fill(attention_mask == 0, 0)
    hid, cache = (prefill_fn or _run_model)(model, input_ids, attention_mask, pos, _new_cache(model))
    if bool((attention_mask[:, -1] == 1).all()):
        cur_hidden = hid[:, -1, :]
    else:
        last = attention_mask.long().sum(-1).clamp_min(1) - 1
        cur_hidden = hid.gather(1, last.view(-1, 1, 1).expand(-1, 1, hid.shape[-1])).squeeze(1)
    cur_logits = torch.nn.functional.linear(cur_hidden, lm_w)
    layers = _cache_layers(cache)
    if repeats > 1:
        layers = [(k.repeat_interleave(repeats, 0).contiguous(), v.repeat_interleave(repeats, 0).contiguous())
                  for k, v in layers]
        cur_hidden = cur_hidden.repeat_interleave(repeats, 0)
        cur_logits = cur_logits.repeat_interleave(repeats, 0)
        attention_mask = attention_mask.repeat_interleave(repeats, 0)
    total = attention_mask.shape[0]
    generated = [[] for _ in range(total)]
    active_ids = list(range(total))
    pending = {}
    full_mask = attention_mask.long()
    logical = full_mask.sum(-1)
    stats = dict(total_acc_length=0, total_decoded_token_num=0, total_verify_rounds=0, total_correction_tokens=0,
                 total_accepted_medusa_tokens=0, total_proposed_medusa_tokens=0)
    # tree / acceptance statistics of the result dict (decoder :1617-1638,
    # accumulated at :2185-2205, :2220, :2250, :2320-2322, :2860)
    nodes_by_head = [0] * min(cfg.num_medusa_heads, len(heads))
    tstat = dict(active_batch_sum=0, tree_node_sum=0.0, tree_sample_count=0, tree_budget_unused=0,
                 tree_query_rows=0, tree_lm_head_rows=0)
    accept_hist, accept_by_depth, proposed_by_depth, layout_counts = {}, {}, {}, {}
    round_idx = 0
    prefill_time = time.perf_counter() - t_start
    while active_ids:
        t_round = time.perf_counter()
        B = len(active_ids)
        remaining = (max_length - logical).tolist()
        old_lens = logical.tolist()
        # root tokens (decoder :1717-1743)
        fresh = [r for r in range(B) if active_ids[r] not in pending]
        root = [0] * B
        if fresh:
            toks = sampler(cur_logits[fresh], [active_ids[r] for r in fresh], round_idx, 0,
                           do_sample=cfg.do_sample, temperature=cfg.temperature,
                           **_cut_kwargs(cfg.top_p, cfg.top_k))
            for r, t in zip(fresh, toks.tolist()):
                root[r] = int(t)
        for r in range(B):
            if active_ids[r] in pending:
                root[r] = pending.pop(active_ids[r])
                stats["total_correction_tokens"] += 1
        plan = plan_tree(active_batch_size=B, num_medusa_heads=cfg.num_medusa_heads, tree_mode=cfg.tree_mode,
                         cpeak_nodes=cfg.cpeak_nodes, min_tree_nodes_per_seq=cfg.min_tree_nodes_per_seq,
                         max_tree_nodes_per_seq=cfg.max_tree_nodes_per_seq, max_tree_depth=cfg.max_tree_depth,
                         fixed_tree_topk_by_depth=list(cfg.fixed_tree_topk_by_depth),
                         adaptive_tree_enabled=cfg.adaptive_tree_enabled,
                         adaptive_min_topk_by_depth=list(cfg.adaptive_min_topk_by_depth))
        n_heads = min(plan.active_heads, len(heads))
        chain = cfg.proposal_mode == "chain"
        projected = project_heads(heads, cur_hidden, n_heads) if not chain else []
        head_logits = (list(torch.nn.functional.linear(torch.cat(projected, 0), lm_w).split(B, 0))
                       if projected else [])
        if cfg.adaptive_tree_enabled and head_logits and plan.topk_by_depth:
            hc = min(len(plan.topk_by_depth), len(head_logits))
            conf = confidences(head_logits[:hc], cfg.adaptive_confidence_metric, cfg.adaptive_confidence_quantile)
            adapted = [topk_from_confidence(c, k, d, adaptive=True, min_topk_by_depth=cfg.adaptive_min_topk_by_depth,
                                            low=cfg.adaptive_confidence_low, high=cfg.adaptive_confidence_high)
                       for d, (k, c) in enumerate(zip(plan.topk_by_depth, conf))]
            adapted = fit_topk_to_budget(adapted, plan.node_budget_per_seq,
                                         min_topk_by_depth=list(cfg.adaptive_min_topk_by_depth)[: len(adapted)],
                                         depth_weight_decay=cfg.adaptive_depth_weight_decay)
            plan = Plan(plan.node_budget_per_seq, len(adapted), adapted, dense_node_count(adapted), plan.mode)
        if chain and plan.topk_by_depth:
            trees = build_chain_trees(root, cur_hidden, plan, heads, cfg.chain_cell, lm_w,
                                      model.get_input_embeddings().weight,
                                      bootstrap_from_medusa=cfg.chain_bootstrap_from_medusa)
        else:
            trees = build_dense_trees(root, head_logits, plan)
        for t in trees:
            stats["total_proposed_medusa_tokens"] += t.node_count - 1
        layout_counts["configured"] = layout_counts.get("configured", 0) + B
        tstat["active_batch_sum"] += B
        tstat["tree_node_sum"] += sum(t.node_count for t in trees) / max(B, 1)
        tstat["tree_sample_count"] += 1
        for t in trees:
            # CandidateTree.nodes_by_head (medusa_tree.py:38-45): nodes per depth >= 2
            for dpt in t.depths:
                if dpt >= 2 and dpt - 2 < len(nodes_by_head):
                    nodes_by_head[dpt - 2] += 1
                if dpt >= 2:
                    proposed_by_depth[dpt] = proposed_by_depth.get(dpt, 0) + 1
            tstat["tree_budget_unused"] += max(0, plan.node_budget_per_seq - t.node_count)
        tree_logits = slots = tree_hidden = None
        if plan.active_heads > 0 and max(t.node_count for t in trees) > 1:
            ids, mask4d, tpos, _ = tree_attention_inputs(trees, full_mask, logical, pad_token_id=pad_token_id,
                                                         dtype=torch.float32)
            tstat["tree_query_rows"] += int(ids.shape[0] * ids.shape[1])
            tcache = _cache_from_layers(model, layers)
            tree_hidden, tcache = _run_model(model, ids, mask4d, tpos, tcache)
            rows, nodes, slots = internal_logit_layout(trees)
            tstat["tree_lm_head_rows"] += len(rows)
            tree_logits = torch.nn.functional.linear(tree_hidden[rows, nodes], lm_w)
            tree_layers = _cache_layers(tcache)
        if tree_logits is None:
            raw_tok = [[r] for r in root]
            raw_nodes = [[0] for _ in trees]
            raw_corr = [None] * B
        else:
            raw_tok, raw_nodes, _, raw_corr = accept_walk_batch(trees, tree_logits, slots, sampler, active_ids,
                                                                round_idx, do_sample=cfg.do_sample,
                                                                temperature=cfg.temperature, top_p=cfg.top_p,
                                                                top_k=cfg.top_k)
        acc, acc_nodes, fin = [], [], []
        for r in range(B):
            tk = raw_tok[r][: max(1, int(remaining[r]))]
            nd = raw_nodes[r][: len(tk)]
            eos = False
            for p, t in enumerate(tk):
                if t == eos_token_id:
                    tk, nd, eos = tk[: p + 1], nd[: p + 1], True
                    break
            done = eos or int(old_lens[r]) + len(tk) >= max_length
            if raw_corr[r] is not None and len(tk) == len(raw_tok[r]) and not done:
                pending[active_ids[r]] = int(raw_corr[r])
            stats["total_acc_length"] += len(tk)
            stats["total_decoded_token_num"] += 1
            stats["total_accepted_medusa_tokens"] += max(len(tk) - 1, 0)
            accept_hist[len(tk)] = accept_hist.get(len(tk), 0) + 1
            for dpt in range(2, len(tk) + 1):
                accept_by_depth[dpt] = accept_by_depth.get(dpt, 0) + 1
            acc.append(tk)
            acc_nodes.append(nd)
            fin.append(done)
            generated[active_ids[r]].extend(tk)
        stats["total_verify_rounds"] += 1
        if record is not None:
            record.append(RoundRecord(trees, plan, acc, acc_nodes, list(raw_corr), dict(pending), fin,
                                      list(active_ids), old_lens,
                                      {"root": list(root), "tree_logits": tree_logits, "slots": slots}))
        max_acc = max(len(t) for t in acc)
        valid_ext = torch.zeros((B, max_acc), dtype=torch.long)
        for r, t in enumerate(acc):
            valid_ext[r, : len(t)] = 1
        if tree_logits is not None:
            layers, _ = extract_path_hf(tree_layers, full_mask.shape[1], acc_nodes)
            last = [p[-1] for p in acc_nodes]
            cur_hidden = tree_hidden[torch.arange(B), torch.tensor(last)]
            cur_logits = torch.stack([
                tree_logits[slots[r][n]] if slots[r][n] >= 0 else torch.nn.functional.linear(cur_hidden[r], lm_w)
                for r, n in enumerate(last)
            ])
            tstat["tree_lm_head_rows"] += sum(1 for r, n in enumerate(last) if slots[r][n] < 0)
        else:
            ids = torch.full((B, max_acc), int(pad_token_id), dtype=torch.long)
            apos = torch.zeros((B, max_acc), dtype=torch.long)
            for r, t in enumerate(acc):
                ids[r, : len(t)] = torch.tensor(t)
                apos[r, : len(t)] = int(old_lens[r]) + torch.arange(len(t))
            new_mask = torch.cat([full_mask, valid_ext], 1)
            hid, c2 = _run_model(model, ids, new_mask, apos, _cache_from_layers(model, layers))
            layers = _cache_layers(c2)
            lastpos = (valid_ext.sum(-1) - 1).clamp_min(0)
            cur_hidden = hid[torch.arange(B), lastpos]
            cur_logits = torch.nn.functional.linear(cur_hidden, lm_w)
        full_mask = torch.cat([full_mask, valid_ext], 1)
        logical = logical + valid_ext.sum(-1)
        keep = [r for r in range(B) if not fin[r]]
        if len(keep) != B:
            if not keep:
                break
            kt = torch.tensor(keep)
            layers = [(k.index_select(0, kt).contiguous(), v.index_select(0, kt).contiguous()) for k, v in layers]
            cur_hidden = cur_hidden.index_select(0, kt)
            cur_logits = cur_logits.index_select(0, kt)
            full_mask = full_mask.index_select(0, kt)
            logical = logical.index_select(0, kt)
            active_ids = [active_ids[r] for r in keep]
        round_idx += 1
        round_times.append((time.perf_counter() - t_round, sum(len(t) for t in acc)))
    decoded = max(stats["total_decoded_token_num"], 1)
    rounds = max(stats["total_verify_rounds"], 1)
    proposed = max(stats["total_proposed_medusa_tokens"], 1)
    stats["average_accept_length"] = stats["total_acc_length"] / decoded
    # the deterministic entries of the reference's result dict (:3039-3117)
    stats.update(
        max_sequence_length=max((len(g) for g in generated), default=0),
        accepted_tokens_per_medusa_step=stats["average_accept_length"],
        total_accepted_draft_tokens=stats["total_accepted_medusa_tokens"],
        total_proposed_draft_tokens=stats["total_proposed_medusa_tokens"],
        correction_token_rate=stats["total_correction_tokens"] / decoded,
        draft_acceptance_rate=stats["total_accepted_medusa_tokens"] / proposed,
        medusa_acceptance_rate=stats["total_accepted_medusa_tokens"] / proposed,
        average_active_batch_size=tstat["active_batch_sum"] / rounds,
        average_tree_nodes_per_seq=tstat["tree_node_sum"] / max(tstat["tree_sample_count"], 1),
        tree_active_heads=max((i + 1 for i, c in enumerate(nodes_by_head) if c > 0), default=0),
        tree_nodes_head1=nodes_by_head[0] if nodes_by_head else 0,
        tree_nodes_head2=nodes_by_head[1] if len(nodes_by_head) > 1 else 0,
        tree_nodes_head3=nodes_by_head[2] if len(nodes_by_head) > 2 else 0,
        tree_total_nodes=sum(nodes_by_head) + stats["total_decoded_token_num"],
        tree_budget_unused=tstat["tree_budget_unused"],
        tree_query_rows=tstat["tree_query_rows"],
        tree_lm_head_rows=tstat["tree_lm_head_rows"],
        tree_lm_head_row_ratio=tstat["tree_lm_head_rows"] / max(tstat["tree_query_rows"], 1),
        accept_length_histogram=accept_hist,
        medusa_accept_by_depth=accept_by_depth,
        medusa_proposed_by_depth=proposed_by_depth,
        actual_tree_layout_counts=layout_counts,
        head3_conditional_path_acceptance=0.0,
        head3_conditional_path_success=0,
        head3_conditional_path_opportunities=0,
        cache_update_mode="extract_path",
        oom_count=0,
        timing_sample_count=0,
    )
    return {"generated_token_ids": generated, **stats, "prefill_time": prefill_time,
            "round_times": round_times}

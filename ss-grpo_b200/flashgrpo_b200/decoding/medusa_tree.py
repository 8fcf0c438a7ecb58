"""Candidate-tree planning (host) and construction (device, K2).

Public names mirror flashgrpo_b200/decoding/medusa_tree.py of the reference:
``CandidateTree``, ``TreePlan``, ``dense_node_count``, ``fit_topk_to_budget``,
``plan_tree`` and ``build_batch_trees`` (dense layout).  Planning is pure
integer arithmetic the host does without touching the device, so the engine
knows each round's tree shape before it launches anything; the device kernel
``fg_build_tree`` computes the same plan (tests check they agree) and builds
the trees, ancestor bits and packed-logit slots for every row in one launch.
The sparse / asymmetric layouts belong to the Reflex/HRDCR subsystem and are
not part of this path.
"""
from __future__ import annotations

import dataclasses
import itertools
import math
from dataclasses import dataclass, field

import torch


@dataclass
class CandidateTree:
    """One row's tree: tokens, parent node ids (-1 for the root), depths (root 1)."""

    tokens: list[int]
    parents: list[int]
    depths: list[int]
    scores: list[float] = field(default_factory=list)

    def __post_init__(self) -> None:
        self.children: dict[int, list[int]] = {}
        for idx, parent in enumerate(self.parents):
            if parent >= 0:
                self.children.setdefault(parent, []).append(idx)

    def ancestors_including_self(self, node_idx: int) -> list[int]:
        chain = [node_idx]
        while self.parents[chain[-1]] >= 0:
            chain.append(self.parents[chain[-1]])
        return chain[::-1]

    @property
    def node_count(self) -> int:
        return len(self.tokens)

    @property
    def nodes_by_head(self) -> list[int]:
        deepest = max((int(d) - 1 for d in self.depths), default=0)
        counts = [0] * deepest
        for d in self.depths:
            if int(d) >= 2:
                counts[int(d) - 2] += 1
        return counts


@dataclass
class TreePlan:
    node_budget_per_seq: int
    active_heads: int
    topk_by_depth: list[int]
    actual_nodes: int
    mode: str
    layout: str = "dense"
    nodes_by_head: list[int] = field(default_factory=list)


def dense_node_count(topk_by_depth) -> int:
    total = width = 1
    for k in topk_by_depth:
        width *= int(k)
        total += width
    return total


def fit_topk_to_budget(topk_by_depth, node_budget, *, min_topk_by_depth=None, depth_weight_decay=0.5):
    """Greedy decrement with the largest nodes-saved / utility-lost ratio
    (utility of branch k at depth d: decay^d * (log(k+1) - log k))."""
    budget = max(1, int(node_budget))
    ks = [max(1, int(k)) for k in topk_by_depth]
    mins = list(min_topk_by_depth or [])
    floors = [max(1, min(ks[d], int(mins[d]) if d < len(mins) else 1)) for d in range(len(ks))]
    weight = max(float(depth_weight_decay), 1e-3)
    while ks and dense_node_count(ks) > budget:
        cur = dense_node_count(ks)
        best = None
        for d, k in enumerate(ks):
            if k <= floors[d]:
                continue
            saved = cur - dense_node_count(ks[:d] + [k - 1] + ks[d + 1:])
            lost = weight ** d * (math.log1p(k) - math.log(k))
            key = (saved / max(lost, 1e-9), saved, d)
            best = key if best is None or key > best else best
        if best is None:
            ks.pop()
            floors.pop()
        else:
            ks[best[2]] -= 1
    return ks


def plan_tree(*, active_batch_size, num_medusa_heads, tree_mode, tree_layout="dense", cpeak_nodes,
              min_tree_nodes_per_seq, max_tree_nodes_per_seq, max_tree_depth, fixed_tree_topk_by_depth,
              adaptive_tree_enabled=False, adaptive_min_topk_by_depth=None, **_unused) -> TreePlan:
    if tree_layout != "dense":
        raise ValueError(f"Unsupported tree_layout={tree_layout} (only 'dense' is on the B200 path)")
    bsz = max(1, int(active_batch_size))
    heads_cap = max(0, int(max_tree_depth) - 1)
    if tree_mode == "fixed":
        budget = int(max_tree_nodes_per_seq)
        ks = [max(1, int(k)) for k in list(fixed_tree_topk_by_depth)[: int(num_medusa_heads)]]
        while ks and dense_node_count(ks) > budget:
            ks[-1] -= 1
            if ks[-1] <= 0:
                ks.pop()
        ks = ks[: min(len(ks), heads_cap)]
    elif tree_mode == "concurrency_aware":
        budget = max(int(min_tree_nodes_per_seq), min(int(max_tree_nodes_per_seq), int(cpeak_nodes) // bsz))
        depth_cap = min(int(num_medusa_heads), heads_cap)
        base = list(fixed_tree_topk_by_depth) or [4, 3, 2, 1, 1]
        ks = []
        if adaptive_tree_enabled:
            mins_in = list(adaptive_min_topk_by_depth or [])
            floor_tree: list[int] = []
            for d in range(depth_cap):
                mk = max(1, int(mins_in[d]) if d < len(mins_in) else 1)
                if dense_node_count(floor_tree + [mk]) > budget:
                    break
                floor_tree.append(mk)
                ks.append(max(mk, int(base[min(d, len(base) - 1)])))
        else:
            width = used = 1
            for d in range(depth_cap):
                room = budget - used
                if room <= 0:
                    break
                k = min(max(1, int(base[min(d, len(base) - 1)])), max(1, room // width))
                if used + width * k > budget:
                    k = room // width
                if k <= 0:
                    break
                ks.append(int(k))
                width *= int(k)
                used += width
    else:
        raise ValueError(f"Unsupported tree_mode={tree_mode}")
    return TreePlan(budget, len(ks), ks, dense_node_count(ks), tree_mode)


def dense_topology(plan: TreePlan, n_heads_available: int | None = None) -> tuple[list[int], list[int]]:
    """Parents and depths of the shared dense tree (BFS, truncated at the budget)."""
    parents, depths = [-1], [1]
    frontier = [0]
    ks = plan.topk_by_depth[: plan.active_heads]
    if n_heads_available is not None:
        ks = ks[:n_heads_available]
    for d, k in enumerate(ks):
        if k <= 0:
            break
        nxt = []
        full = False
        for p in frontier:
            for _ in range(int(k)):
                parents.append(p)
                depths.append(d + 2)
                nxt.append(len(parents) - 1)
                if len(parents) >= plan.node_budget_per_seq:
                    full = True
                    break
            if full:
                break
        frontier = nxt
        if not frontier or len(parents) >= plan.node_budget_per_seq:
            break
    return parents, depths


def internal_nodes(parents: list[int]) -> list[int]:
    has_child = set(p for p in parents if p >= 0)
    return [i for i in range(len(parents)) if i in has_child]


def max_adaptive_internal(plan: TreePlan, n_heads_available: int | None = None) -> int:
    """Most internal nodes that any adaptive tree of this base plan can have.

    Adaptive top-k (flash_medusa_decoder.py:1021-1095) keeps every depth's
    width in [1, base width] and may drop trailing depths; the tree is then
    expanded in BFS order up to the node budget.  A narrower, deeper tree can
    have more internal nodes than the base plan's own (e.g. a 16-node budget:
    base (4, 3, 2) has 5 internal nodes, (4, 1, 1) has 9), so buffers of
    internal-node rows are sized by this bound.  Every width vector is tried
    (few: the product of the base widths); past 4096 of them the bound is
    the node budget - 1."""
    ks = [int(k) for k in plan.topk_by_depth[: plan.active_heads]]
    if n_heads_available is not None:
        ks = ks[:n_heads_available]
    ks = [k for k in ks if k > 0]
    if math.prod(ks) * max(len(ks), 1) > 4096:
        return max(plan.node_budget_per_seq - 1, 1)
    best = len(internal_nodes(dense_topology(plan, n_heads_available)[0]))
    for depth in range(1, len(ks) + 1):
        for widths in itertools.product(*[range(1, k + 1) for k in ks[:depth]]):
            p = dataclasses.replace(plan, active_heads=depth, topk_by_depth=list(widths))
            best = max(best, len(internal_nodes(dense_topology(p)[0])))
    return best


def build_batch_trees(root_tokens: torch.Tensor, medusa_logits: list[torch.Tensor], plan: TreePlan,
                      **_unused) -> list[CandidateTree]:
    """API mirror of the reference builder: candidates by the device top-k
    (ties -> lower index), trees assembled by the K2 kernel, returned as
    CandidateTree objects for callers that want Python structures."""
    from .. import ops

    n_heads = min(plan.active_heads, len(medusa_logits))
    root = root_tokens.to(torch.int32).contiguous()
    B = root.shape[0]
    kmax = max([int(k) for k in plan.topk_by_depth[:n_heads]] + [1])
    cands = [ops.row_topk(lg, kmax) for lg in medusa_logits[:n_heads]]
    cand_idx = torch.stack([c[0] for c in cands]) if cands else None
    params = ops.plan_params(tree_mode="explicit", active_batch_size=B, num_medusa_heads=n_heads, cpeak_nodes=0,
                             min_tree_nodes_per_seq=1, max_tree_nodes_per_seq=plan.node_budget_per_seq,
                             max_tree_depth=n_heads + 1, fixed_tree_topk_by_depth=plan.topk_by_depth[:n_heads])
    nmax = max(plan.node_budget_per_seq, 2)
    out = ops.build_tree(params, root, cand_idx, None, None, None, nmax=min(nmax, 128),
                         logits_dtype=medusa_logits[0].dtype if medusa_logits else torch.float32,
                         row_len=torch.zeros(B, dtype=torch.int32, device=root.device))
    n = int(out["plan"][10])
    tokens = out["tokens"][:, :n].tolist()
    parents = out["parents"][:n].tolist()
    depths = out["depths"][:n].tolist()
    return [CandidateTree(tokens=tokens[b], parents=list(parents), depths=list(depths)) for b in range(B)]

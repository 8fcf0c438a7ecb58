"""FlashMedusaDecoder: the speculative rollout loop, B200 edition.

Drop-in for flashgrpo_b200/decoding/flash_medusa_decoder.py of the reference:
same ``FlashMedusaConfig`` knobs for this path, same constructor checks
(:227-251), same ``generate(...)`` signature (:1272-1283) and result keys
(:3039-3117).  Each round runs on the GPU through ``VerifyEngine`` (K1-K4
behind the C ABI); the host only plans the tree shape, replays the round's
CUDA graph and reads back the accepted tokens.

Sampling: draws come from Philox uniforms indexed by (sequence id, round,
draw) and the fg-icdf-v1 inverse CDF, so a seeded run is reproducible bit for
bit.  Nucleus (``top_p < 1``) and top-k sampling (fg-icdf-v1n / v1k: the
reference's kept sets on exact integer masses), adaptive trees and chain
proposals are supported; ``cache_update_mode="recompute_accepted"``,
the sparse tree layouts, adaptive widths with chain proposals and the
Reflex/HRDCR machinery are not on this path and are rejected explicitly.

Result timings.  A round is one CUDA graph, so the reference's per-phase host
timers (proposal, tree verify, cache update) become CUDA events at the phase
boundaries inside the graph: proposal + tree build | verify forward +
internal-node lm_head | acceptance + extract_path.  Every
``metrics_timing_sample_interval``-th round is timed that way (the sampled
``*_cuda_time_s`` keys, as the reference samples, :1816-1822, :2940-2946);
with ``statistical_time=True`` every round is, and the ``*_time_cost`` keys
are the sums of the measured phase times.  Without it they split the rounds'
host-measured wall time by the phase shares of the sampled rounds.
"""
from __future__ import annotations

import math
import time
import warnings
import dataclasses
from dataclasses import dataclass

import torch

from .. import ops
from ..engine.verify import DecodeState, RoundConfig, VerifyEngine, unwrap_causal_lm
from .medusa_tree import dense_node_count, plan_tree


@dataclass
class FlashMedusaConfig:
    num_medusa_heads: int = 3
    tree_mode: str = "concurrency_aware"
    tree_layout: str = "dense"
    acceptance: str = "exact_target"
    cache_update_mode: str = "extract_path"
    allow_recompute_fallback: bool = True
    cpeak_nodes: int = 512
    min_tree_nodes_per_seq: int = 1
    max_tree_nodes_per_seq: int = 10
    max_tree_depth: int = 4
    fixed_tree_topk_by_depth: tuple[int, ...] = (4, 3, 2)
    do_sample: bool = True
    temperature: float = 1.0
    top_p: float = 0.95
    top_k: int | None = None
    clone_tree_cache: bool = True
    proposal_mode: str = "medusa"
    chain_enable_after: int = 0
    chain_bootstrap_from_medusa: bool = True
    enable_medusa_spec_after: int = 0
    adaptive_tree_enabled: bool = False
    adaptive_confidence_metric: str = "top1_prob"
    adaptive_confidence_quantile: float = 0.25
    adaptive_confidence_low: float = 0.15
    adaptive_confidence_high: float = 0.45
    adaptive_min_topk_by_depth: tuple[int, ...] = (1, 1, 1)
    adaptive_depth_weight_decay: float = 0.5
    head_inference_autocast: bool = True
    project_internal_tree_logits_only: bool = True
    inplace_kv_compaction: bool = True
    reflex_enabled: bool = False
    metrics_timing_sample_interval: int = 32
    # B200 engine knobs (no counterpart in the reference)
    sampling_seed: int = 0
    use_cuda_graphs: bool = True
    attention_splits: int = 0
    # proposal lm_head: "separate" (cuBLAS + fg_row_topk; measured faster on B200, 3.60 vs 3.66 ms per
    # config-2 round) or "fused" (tcgen05 GEMM with the top-k in its epilogue)
    lm_head_kernel: str = "separate"
    # verify projections + internal lm_head: "auto" (per shape, fg_linear or cuBLAS, whichever
    # measured faster), "native" (fg_linear, tcgen05, always) or "cublas"
    dense_kernel: str = "auto"
    autotune_dense: bool = True    # time fg_linear's tilings once per projection shape


class FlashMedusaDecoder:
    def __init__(self, target_model, medusa_heads, tokenizer, config: FlashMedusaConfig):
        self.target_model = target_model
        self.medusa_heads = medusa_heads
        self.tokenizer = tokenizer
        self.config = config
        if config.acceptance != "exact_target":
            raise NotImplementedError("Only exact_target acceptance is implemented in the main FlashGRPO path")
        if config.cache_update_mode not in {"extract_path", "recompute_accepted"}:
            raise ValueError(f"Unsupported cache_update_mode={config.cache_update_mode}")
        if config.cache_update_mode != "extract_path":
            raise NotImplementedError("cache_update_mode='recompute_accepted' is not on the B200 path: the accepted "
                                      "K/V are compacted from the tree cache (extract_path) on the device")
        if config.proposal_mode not in {"medusa", "chain"}:
            raise ValueError(f"Unsupported proposal_mode={config.proposal_mode}")
        if config.proposal_mode == "chain" and config.adaptive_tree_enabled:
            raise NotImplementedError("adaptive widths for chain proposals are not on the B200 path")
        if config.tree_layout != "dense":
            raise NotImplementedError("sparse tree layouts belong to the Reflex/HRDCR subsystem (tree_layout='dense')")
        if config.reflex_enabled:
            raise NotImplementedError("Reflex/HRDCR proposal adaptation is not on the B200 path")
        if config.lm_head_kernel not in {"fused", "separate"}:
            raise ValueError(f"Unsupported lm_head_kernel={config.lm_head_kernel}")
        if config.dense_kernel not in {"auto", "native", "cublas"}:
            raise ValueError(f"Unsupported dense_kernel={config.dense_kernel}")
        self._engine: VerifyEngine | None = None
        # captured round graphs, keyed by (state, round shape, round config);
        # a shape is run eagerly once before it is captured
        self._graphs: dict = {}
        self._seen: set = set()

    # ------------------------------------------------------------- helpers
    @property
    def engine(self) -> VerifyEngine:
        if self._engine is None:
            self._engine = VerifyEngine(self.target_model, self.medusa_heads,
                                        autotune=bool(self.config.autotune_dense), dense=self.config.dense_kernel)
        return self._engine

    def _plan(self, active: int):
        cfg = self.config
        return plan_tree(active_batch_size=active, num_medusa_heads=min(cfg.num_medusa_heads,
                                                                        len(self.engine.heads)),
                         tree_mode=cfg.tree_mode, tree_layout=cfg.tree_layout, cpeak_nodes=cfg.cpeak_nodes,
                         min_tree_nodes_per_seq=cfg.min_tree_nodes_per_seq,
                         max_tree_nodes_per_seq=cfg.max_tree_nodes_per_seq, max_tree_depth=cfg.max_tree_depth,
                         fixed_tree_topk_by_depth=list(cfg.fixed_tree_topk_by_depth),
                         adaptive_tree_enabled=bool(cfg.adaptive_tree_enabled),
                         adaptive_min_topk_by_depth=list(cfg.adaptive_min_topk_by_depth))

    def _params(self, active: int):
        cfg = self.config
        return ops.plan_params(
            tree_mode=cfg.tree_mode, active_batch_size=active,
            num_medusa_heads=min(cfg.num_medusa_heads, len(self.engine.heads)), cpeak_nodes=cfg.cpeak_nodes,
            min_tree_nodes_per_seq=cfg.min_tree_nodes_per_seq, max_tree_nodes_per_seq=cfg.max_tree_nodes_per_seq,
            max_tree_depth=cfg.max_tree_depth, fixed_tree_topk_by_depth=cfg.fixed_tree_topk_by_depth,
            adaptive_tree_enabled=bool(cfg.adaptive_tree_enabled),
            adaptive_min_topk_by_depth=tuple(cfg.adaptive_min_topk_by_depth),
            adaptive_confidence_metric=cfg.adaptive_confidence_metric,
            adaptive_confidence_quantile=cfg.adaptive_confidence_quantile,
            adaptive_confidence_low=cfg.adaptive_confidence_low, adaptive_confidence_high=cfg.adaptive_confidence_high,
            adaptive_depth_weight_decay=cfg.adaptive_depth_weight_decay)

    def round_config(self, max_length: int, generation_step: int = 0) -> RoundConfig:
        cfg = self.config
        chain = cfg.proposal_mode == "chain" and int(generation_step) >= int(cfg.chain_enable_after)
        if chain and self.engine.heads.chain is None:
            raise ValueError("proposal_mode='chain' needs a ChainDraftCell (chain_cell.*) in the MEDUSA heads")
        eos = getattr(self.tokenizer, "eos_token_id", None)
        pad = getattr(self.tokenizer, "pad_token_id", None)
        eos = eos if eos is not None else (pad if pad is not None else 0)
        top_p = 1.0 if cfg.top_p is None else float(cfg.top_p)
        # the reference cuts only for 0 < top_k < vocab (acceptance.py:68); so do the kernels
        top_k = 0 if cfg.top_k is None else int(cfg.top_k)
        return RoundConfig(do_sample=bool(cfg.do_sample), temperature=float(cfg.temperature), top_p=top_p,
                           top_k=top_k, eos_id=int(eos),
                           max_length=int(max_length), seed=int(cfg.sampling_seed),
                           attn_splits=int(cfg.attention_splits), lm_head=str(cfg.lm_head_kernel),
                           dense=str(cfg.dense_kernel), chain=chain,
                           chain_bootstrap=bool(cfg.chain_bootstrap_from_medusa))

    def max_heads(self) -> int:
        cfg = self.config
        return max(0, min(cfg.num_medusa_heads, len(self.engine.heads), cfg.max_tree_depth - 1))

    # ------------------------------------------------------------ generate
    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, attention_mask: torch.Tensor, *, repeated_generate_nums=None,
                 max_length: int = 2048, statistical_time: bool = False, generation_step: int = 0,
                 collect_reflex_aux_cache=None, persistent_reflex_memory=None) -> dict:
        cfg = self.config
        eng = self.engine
        repeats = max(1, int(repeated_generate_nums or 1))
        dev = eng.device
        total_start = time.time()
        n_heads = self.max_heads()
        capacity = int(max_length) + max(int(cfg.max_tree_nodes_per_seq), 1) + 2
        torch.cuda.synchronize(dev)
        t0 = time.time()
        st = eng.prefill(input_ids, attention_mask, repeats=repeats, capacity=capacity, n_heads=n_heads)
        torch.cuda.synchronize(dev)
        prefill_time = time.time() - t0
        rcfg = self.round_config(max_length, generation_step)
        B = st.B
        generated = [[] for _ in range(B)]
        active_host = [True] * B
        row_len_host = st.row_len.tolist()
        acc = RolloutStats(min(cfg.num_medusa_heads, len(eng.heads)))
        pending_host = [-1] * B
        graphs, seen = self._graphs, self._seen
        rcfg_key = dataclasses.astuple(rcfg)
        setups: dict = {}
        flat_bufs: dict = {}
        interval = max(1, int(cfg.metrics_timing_sample_interval))
        timer = self._phase_events(dev)
        use_tree = int(generation_step) >= int(cfg.enable_medusa_spec_after)

        rows_sent: set = set()
        pinned = [None, None]  # round outputs, alternating between consecutive rounds
        n_launched = 0
        # (row count, timed) -> (captured graph, output parts, flat buffer):
        # the steady-state launch replays and enqueues the copy with no lookups
        fast: dict = {}

        def launch(act_rows):
            """Enqueue one round over act_rows and the copy of its outputs to
            pinned host memory; returns what processing the round needs."""
            nonlocal n_launched
            n_active = len(act_rows)
            timed = bool(statistical_time) or n_launched % interval == 0
            f = fast.get((n_active, timed))
            if f is not None:
                tv = time.time()
                f[0].replay()
                host = copy_out(f[1], f[2])
                return (act_rows, *setups[n_active][:4], timed, tv, host)
            setup = setups.get(n_active)
            if setup is None:
                plan = self._plan(n_active)
                if not use_tree:
                    plan.topk_by_depth, plan.active_heads = [], 0
                nh = min(n_heads, plan.active_heads)
                plan.topk_by_depth = plan.topk_by_depth[:nh]
                plan.active_heads = nh
                adaptive = bool(cfg.adaptive_tree_enabled) and nh > 0
                params = self._params(n_active) if nh > 0 else ops.plan_params(
                    tree_mode="explicit", active_batch_size=n_active, num_medusa_heads=0, cpeak_nodes=0,
                    min_tree_nodes_per_seq=1, max_tree_nodes_per_seq=1, max_tree_depth=1,
                    fixed_tree_topk_by_depth=())
                setup = setups[n_active] = (plan, nh, nh + 2, adaptive, params)
            plan, nh, dcap, adaptive, params = setup
            if n_active < B:
                rs = eng.view(st, n_active, n_heads)
                # finished rows only ever leave, so a row count names one row
                # set within a call: its map is sent once
                if n_active not in rows_sent:
                    rows_host = torch.tensor(act_rows, dtype=torch.int32).pin_memory()
                    rs.rows.copy_(rows_host, non_blocking=True)
                    rows_sent.add(n_active)
            else:
                rs = st
            rb = eng.buffers(n_active, plan, nh, dcap, adaptive=adaptive)
            # CUDA events at the phase boundaries on sampled rounds (every
            # round with statistical_time)
            ev = timer if timed else None
            key = (id(rs), n_active, rb.N, tuple(plan.topk_by_depth), plan.node_budget_per_seq, adaptive, rcfg_key,
                   timed)
            tv = time.time()
            if cfg.use_cuda_graphs and key in seen:
                if key not in graphs:
                    graphs[key] = (eng.graph_round(rs, rb, params, rcfg, phase_events=ev), params)
                graphs[key][0].replay()
            else:
                eng.run_round(rs, rb, params, rcfg, phase_events=ev)
                seen.add(key)
            out = rb.out
            parts = [out["acc_len"], out["finished"], rs.pending, out["last_node"], rb.tree["plan"],
                     out["acc_tokens"].view(-1)]
            fb = flat_bufs.get((id(rb), id(rs)))
            if fb is None:
                fb = flat_bufs[(id(rb), id(rs))] = torch.empty(sum(t.numel() for t in parts), dtype=torch.int32,
                                                              device=dev)
            if cfg.use_cuda_graphs and key in graphs and (n_active == B or n_active in rows_sent):
                fast[(n_active, timed)] = (graphs[key][0], parts, fb)
            host = copy_out(parts, fb)
            return act_rows, plan, nh, dcap, adaptive, timed, tv, host

        def copy_out(parts, fb):
            """The round's outputs gathered into one device buffer and copied
            to this round's pinned host buffer (a numpy view of it)."""
            nonlocal n_launched
            torch.cat(parts, out=fb)
            slot = n_launched & 1
            if pinned[slot] is None or pinned[slot].numel() < fb.numel():
                pinned[slot] = torch.empty(fb.numel(), dtype=torch.int32, pin_memory=True)
            host = pinned[slot][: fb.numel()]
            host.copy_(fb, non_blocking=True)
            n_launched += 1
            return host.numpy()

        def process(rnd, wall, phases):
            """Host bookkeeping of a finished round (tokens, statistics); runs
            while the next round executes on the device."""
            act_rows, plan, nh, dcap, adaptive, _, _, vals = rnd
            Br = len(act_rows)  # outputs are per round row: round row i is state row act_rows[i]
            acc_len = vals[:Br].tolist()
            pend = vals[2 * Br:3 * Br].tolist()
            last = vals[3 * Br:4 * Br].tolist()
            plan_dev = vals[4 * Br:4 * Br + 16].tolist()
            toks = vals[4 * Br + 16:]
            # the round's tree as built on the device (adaptive rounds may be smaller)
            topk_round = plan_dev[2:2 + plan_dev[1]] if nh > 0 else []
            n_tree = plan_dev[10] if nh > 0 else 1
            if nh > 0 and n_tree <= 1 and not cfg.allow_recompute_fallback:
                # the reference's verify needs a tree cache to extract from (:2881-2882)
                raise RuntimeError("KV extraction was requested but no tree cache was available")
            acc.round(Br, plan.node_budget_per_seq, topk_round, n_tree, last, use_tree, nh, wall, phases)
            acc.last_plan = {"B_cur": Br, "node_budget_per_seq": plan.node_budget_per_seq,
                             "active_heads": plan.active_heads, "topk_by_depth": list(topk_round),
                             "actual_nodes": n_tree, "proposal_mode": "chain" if rcfg.chain else "medusa",
                             "adaptive_tree": {"topk": list(topk_round)} if adaptive else {},
                             "nodes_by_head": tree_level_counts(topk_round, n_tree)}
            pend_before = [pending_host[r] for r in act_rows]
            for i, row in enumerate(act_rows):
                row_len_host[row] += acc_len[i]
                pending_host[row] = pend[i]
                generated[row].extend(toks[i * dcap: i * dcap + acc_len[i]].tolist())
            acc.rows(acc_len, pend_before)

        # One round in flight ahead of the host: as soon as a round's outputs
        # are on the host, the next round (whose row set depends only on the
        # finished flags) is launched, and the finished round's tokens and
        # statistics are processed while it runs.
        cur = launch([r for r in range(B) if active_host[r]])
        while cur is not None:
            torch.cuda.current_stream(dev).synchronize()
            wall = time.time() - cur[6]
            phases = [timer[i].elapsed_time(timer[i + 1]) / 1000.0 for i in range(3)] if cur[5] else None
            vals = cur[7]
            Br = len(cur[0])
            fin = vals[Br:2 * Br]
            act_rows = cur[0]
            if fin.any():
                for i in fin.nonzero()[0].tolist():
                    active_host[cur[0][i]] = False
                act_rows = [r for r in cur[0] if active_host[r]]
            nxt = launch(act_rows) if act_rows else None
            process(cur, wall, phases)
            cur = nxt
        return acc.result(generated, prefill_time=prefill_time, total_time=time.time() - total_start,
                          statistical_time=bool(statistical_time), cache_update_mode=cfg.cache_update_mode)

    def _phase_events(self, dev):
        """Four timing events (graph-capturable) at the round's phase boundaries."""
        ev = getattr(self, "_timer", None)
        if ev is None:
            ev = self._timer = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(4)]
        return ev


def tree_level_counts(topk_by_depth, n_nodes: int) -> list[int]:
    """Nodes per depth below the root of the dense tree with these widths,
    expanded breadth first and cut at n_nodes (CandidateTree.nodes_by_head,
    medusa_tree.py:38-45, for the shared topology of a round)."""
    counts, total, width = [], 1, 1
    for k in topk_by_depth:
        width *= int(k)
        c = min(width, n_nodes - total)
        if c <= 0:
            break
        counts.append(c)
        total += c
        width = c
    return counts


def tree_internal_nodes(topk_by_depth, n_nodes: int) -> set[int]:
    """Node ids with children in that tree (BFS order: a level's nodes with
    children are its first ceil(children / width) nodes)."""
    counts = tree_level_counts(topk_by_depth, n_nodes)
    internal, start = set(), 0
    level = [1] + counts
    for d, k in enumerate(topk_by_depth[: len(counts)]):
        n_par = -(-counts[d] // int(k))
        internal.update(range(start, start + n_par))
        start += level[d]
    return internal


class RolloutStats:
    """The statistics of the reference's generate result dict
    (flash_medusa_decoder.py:1617-1638 accumulated at :2185-2205, :2220,
    :2250, :2316-2326, :2860; assembled at :3039-3117), from the per-round
    outputs the engine reads back: every row of a round shares the tree's
    topology, so per-tree counts are per-round counts times the active rows."""

    def __init__(self, n_stat_heads: int):
        self.nodes_by_head = [0] * n_stat_heads
        self.rounds = 0
        self.c = dict(total_acc_length=0, total_decoded_token_num=0, total_verify_rounds=0,
                      total_correction_tokens=0, total_accepted_medusa_tokens=0, total_proposed_medusa_tokens=0)
        self.active_batch_sum = 0
        self.tree_node_sum = 0.0
        self.tree_budget_unused = 0
        self.tree_query_rows = 0
        self.tree_lm_head_rows = 0
        self.extract_ok = 0
        self.extract_fallback = 0
        self.accept_hist: dict[int, int] = {}
        self.accept_by_depth: dict[int, int] = {}
        self.proposed_by_depth: dict[int, int] = {}
        self.layouts: dict[str, int] = {}
        self.last_plan: dict = {}
        self.n_tree_round: list[int] = []
        # timings: host wall time of every round, device phase times of the timed ones
        self.wall = 0.0
        self.wall_timed = 0.0
        self.phase = [0.0, 0.0, 0.0]
        self.sampled = [0.0, 0.0, 0.0]
        self.samples = 0

    def round(self, n_active, budget, topk_round, n_tree, last_nodes, use_tree, nh, wall, phases):
        self.rounds += 1
        self.c["total_verify_rounds"] += 1
        self.active_batch_sum += n_active
        self.tree_node_sum += n_tree
        self.n_tree_round.append(n_tree)
        if use_tree:
            self.layouts["configured"] = self.layouts.get("configured", 0) + n_active
        counts = tree_level_counts(topk_round, n_tree)
        for h, c in enumerate(counts[: len(self.nodes_by_head)]):
            self.nodes_by_head[h] += c * n_active
        for d, c in enumerate(counts):
            self.proposed_by_depth[d + 2] = self.proposed_by_depth.get(d + 2, 0) + c * n_active
        self.tree_budget_unused += max(0, int(budget) - n_tree) * n_active
        if nh > 0 and n_tree > 1:
            # a tree verify ran: query rows, packed internal-node logits and
            # the leaf rows whose next logits the lm_head recomputes
            internal = tree_internal_nodes(topk_round, n_tree)
            self.tree_query_rows += n_active * n_tree
            self.tree_lm_head_rows += n_active * len(internal) + sum(1 for n in last_nodes if n not in internal)
            self.extract_ok += 1
        elif nh > 0:
            self.extract_fallback += 1
        self.wall += wall
        if phases is not None:
            self.samples += 1
            self.wall_timed += wall
            for i in range(3):
                self.sampled[i] += phases[i]

    def rows(self, acc_len, pend_before):
        n_tree = self.n_tree_round.pop(0)
        for a, p in zip(acc_len, pend_before):
            if p >= 0:
                self.c["total_correction_tokens"] += 1
            self.c["total_acc_length"] += a
            self.c["total_decoded_token_num"] += 1
            self.c["total_accepted_medusa_tokens"] += max(a - 1, 0)
            self.c["total_proposed_medusa_tokens"] += max(n_tree - 1, 0)
            self.accept_hist[a] = self.accept_hist.get(a, 0) + 1
            for d in range(2, a + 1):
                self.accept_by_depth[d] = self.accept_by_depth.get(d, 0) + 1

    def result(self, generated, *, prefill_time, total_time, statistical_time, cache_update_mode) -> dict:
        c = self.c
        rounds = max(c["total_verify_rounds"], 1)
        decoded = max(c["total_decoded_token_num"], 1)
        proposed = max(c["total_proposed_medusa_tokens"], 1)
        avg_accept = c["total_acc_length"] / decoded
        if statistical_time:
            head_t, verify_t, update_t = self.sampled
        else:
            # the rounds' wall time, split by the sampled rounds' phase shares
            tot = sum(self.sampled)
            share = [x / tot for x in self.sampled] if tot > 0 else [0.0, 1.0, 0.0]
            head_t, verify_t, update_t = (self.wall * x for x in share)
        nbh = self.nodes_by_head
        total_tokens = sum(len(g) for g in generated)
        return {
            "generated_token_ids": generated,
            "max_sequence_length": max((len(g) for g in generated), default=0),
            **c,
            "average_accept_length": float(avg_accept),
            "accepted_tokens_per_medusa_step": float(avg_accept),
            "total_accepted_draft_tokens": c["total_accepted_medusa_tokens"],
            "total_proposed_draft_tokens": c["total_proposed_medusa_tokens"],
            "correction_token_rate": c["total_correction_tokens"] / decoded,
            "draft_acceptance_rate": c["total_accepted_medusa_tokens"] / proposed,
            "medusa_acceptance_rate": c["total_accepted_medusa_tokens"] / proposed,
            "average_active_batch_size": self.active_batch_sum / rounds,
            "average_tree_nodes_per_seq": self.tree_node_sum / rounds,
            "tree_active_heads": max((i + 1 for i, n in enumerate(nbh) if n > 0), default=0),
            "tree_nodes_head1": nbh[0] if nbh else 0,
            "tree_nodes_head2": nbh[1] if len(nbh) > 1 else 0,
            "tree_nodes_head3": nbh[2] if len(nbh) > 2 else 0,
            "tree_total_nodes": sum(nbh) + c["total_decoded_token_num"],
            "tree_budget_unused": self.tree_budget_unused,
            "tree_query_rows": self.tree_query_rows,
            "tree_lm_head_rows": self.tree_lm_head_rows,
            "tree_lm_head_row_ratio": self.tree_lm_head_rows / max(self.tree_query_rows, 1),
            "accept_length_histogram": self.accept_hist,
            "medusa_accept_by_depth": self.accept_by_depth,
            "medusa_proposed_by_depth": self.proposed_by_depth,
            "last_tree_plan": self.last_plan,
            "actual_tree_layout_counts": self.layouts,
            # the head-3 gate statistics exist only with the Reflex/HRDCR manager
            "head3_conditional_path_acceptance": 0.0,
            "head3_conditional_path_success": 0,
            "head3_conditional_path_opportunities": 0,
            "cache_update_mode": cache_update_mode,
            "kv_extraction_success_count": self.extract_ok,
            "kv_extraction_fallback_count": self.extract_fallback,
            "kv_extraction_time": update_t,
            "recompute_fallback_time": 0.0,
            "oom_count": 0,
            "total_time_cost": total_time,
            "prefill_time_cost": prefill_time,
            "target_time_cost": prefill_time + verify_t + update_t,
            "tree_verify_time_cost": verify_t,
            "cache_update_time_cost": update_t,
            "medusa_head_time_cost": head_t,
            "sampled_medusa_head_cuda_time_s": self.sampled[0],
            "sampled_tree_verify_cuda_time_s": self.sampled[1],
            "timing_sample_count": self.samples,
            "draft_time_cost": head_t,
            "check_time_cost": 0.0,
            "tokens_per_sec_generation": total_tokens / max(total_time, 1e-9),
            "reflex_metrics": {"enabled": False},
            "reflex_head_metrics": {},
            "reflex_aux_records": {},
            "persistent_memory_feedback": {},
            "motivation_trace": [],
        }

"""FlashMedusaDecoder: the speculative rollout loop, B200 edition.

Drop-in for flashgrpo_b200/decoding/flash_medusa_decoder.py of the reference:
same ``FlashMedusaConfig`` knobs for this path, same constructor checks
(:227-251), same ``generate(...)`` signature (:1272-1283) and result keys
(:3039-3117).  Each round runs on the GPU through ``VerifyEngine`` (K1-K4
behind the C ABI); the host only plans the tree shape, replays the round's
CUDA graph and reads back the accepted tokens.

Sampling: draws come from Philox uniforms indexed by (sequence id, round,
draw) and the fg-icdf-v1 inverse CDF, so a seeded run is reproducible bit for
bit.  Nucleus sampling (``top_p < 1``), adaptive trees and chain proposals
are supported; ``top_k`` sampling, the sparse tree layouts, adaptive widths
with chain proposals and the Reflex/HRDCR machinery are not on this path and
are rejected explicitly.
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
    lm_head_kernel: str = "fused"  # "fused" (tcgen05 + top-k epilogue) or "separate" (cuBLAS + fg_row_topk)


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
        if config.proposal_mode not in {"medusa", "chain"}:
            raise ValueError(f"Unsupported proposal_mode={config.proposal_mode}")
        if config.proposal_mode == "chain" and config.adaptive_tree_enabled:
            raise NotImplementedError("adaptive widths for chain proposals are not on the B200 path")
        if config.tree_layout != "dense":
            raise NotImplementedError("sparse tree layouts belong to the Reflex/HRDCR subsystem (tree_layout='dense')")
        if config.reflex_enabled:
            raise NotImplementedError("Reflex/HRDCR proposal adaptation is not on the B200 path")
        if config.top_k is not None:
            raise NotImplementedError("top_k sampling is not on the B200 path yet")
        if config.lm_head_kernel not in {"fused", "separate"}:
            raise ValueError(f"Unsupported lm_head_kernel={config.lm_head_kernel}")
        self._engine: VerifyEngine | None = None
        # captured round graphs, keyed by (state, round shape, round config);
        # a shape is run eagerly once before it is captured
        self._graphs: dict = {}
        self._seen: set = set()

    # ------------------------------------------------------------- helpers
    @property
    def engine(self) -> VerifyEngine:
        if self._engine is None:
            self._engine = VerifyEngine(self.target_model, self.medusa_heads)
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
        return RoundConfig(do_sample=bool(cfg.do_sample), temperature=float(cfg.temperature), top_p=top_p,
                           eos_id=int(eos),
                           max_length=int(max_length), seed=int(cfg.sampling_seed),
                           attn_splits=int(cfg.attention_splits), lm_head=str(cfg.lm_head_kernel), chain=chain,
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
        stats = dict(total_acc_length=0, total_decoded_token_num=0, total_verify_rounds=0,
                     total_correction_tokens=0, total_accepted_medusa_tokens=0, total_proposed_medusa_tokens=0)
        accept_hist: dict[int, int] = {}
        accept_by_depth: dict[int, int] = {}
        active_batch_sum = 0
        tree_node_sum = 0.0
        tree_plan_last = {}
        pending_host = [-1] * B
        graphs, seen = self._graphs, self._seen
        pinned = None
        verify_time = 0.0
        rcfg_key = dataclasses.astuple(rcfg)
        setups: dict = {}
        flat_bufs: dict = {}

        def account(d):
            """Host bookkeeping of a finished round (tokens, statistics); runs
            while the next round executes on the device."""
            rows_d, acc_d, toks_d, dcap_d, n_tree_d, pend_before = d
            for i, r in enumerate(rows_d):
                if pend_before[i] >= 0:
                    stats["total_correction_tokens"] += 1
                a = acc_d[i]
                generated[r].extend(toks_d[i * dcap_d: i * dcap_d + a])
                stats["total_acc_length"] += a
                stats["total_decoded_token_num"] += 1
                stats["total_accepted_medusa_tokens"] += max(a - 1, 0)
                stats["total_proposed_medusa_tokens"] += max(n_tree_d - 1, 0)
                accept_hist[a] = accept_hist.get(a, 0) + 1
                for d_ in range(2, a + 1):
                    accept_by_depth[d_] = accept_by_depth.get(d_, 0) + 1

        deferred = None
        while any(active_host):
            # finished rows retire: the round runs on the active rows only
            # (select_cache_batch semantics), through a row map into the
            # cache when some rows have finished
            act_rows = [r for r in range(B) if active_host[r]]
            n_active = len(act_rows)
            setup = setups.get(n_active)
            if setup is None:
                use_tree = int(generation_step) >= int(cfg.enable_medusa_spec_after)
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
                rows_host = torch.tensor(act_rows, dtype=torch.int32).pin_memory()
                rs.rows.copy_(rows_host, non_blocking=True)
            else:
                rs = st
            rb = eng.buffers(n_active, plan, nh, dcap, adaptive=adaptive)
            key = (id(rs), n_active, rb.N, tuple(plan.topk_by_depth), plan.node_budget_per_seq, adaptive, rcfg_key)
            tv = time.time()
            if cfg.use_cuda_graphs and key in seen:
                if key not in graphs:
                    graphs[key] = (eng.graph_round(rs, rb, params, rcfg), params)
                graphs[key][0].replay()
            else:
                eng.run_round(rs, rb, params, rcfg)
                seen.add(key)
            out = rb.out
            parts = [out["acc_len"], out["finished"], rs.pending, rb.tree["plan"], out["acc_tokens"].view(-1)]
            fb = flat_bufs.get((id(rb), id(rs)))
            if fb is None:
                fb = flat_bufs[(id(rb), id(rs))] = torch.empty(sum(t.numel() for t in parts), dtype=torch.int32,
                                                              device=dev)
            torch.cat(parts, out=fb)
            if pinned is None or pinned.numel() < fb.numel():
                pinned = torch.empty(fb.numel(), dtype=torch.int32, pin_memory=True)
            host = pinned[: fb.numel()]
            host.copy_(fb, non_blocking=True)
            if deferred is not None:
                account(deferred)
                deferred = None
            torch.cuda.current_stream(dev).synchronize()
            verify_time += time.time() - tv
            vals = host.tolist()
            Br = n_active  # outputs are per round row: round row i is state row act_rows[i]
            acc_len = vals[:Br]
            fin = vals[Br:2 * Br]
            pend = vals[2 * Br:3 * Br]
            plan_dev = vals[3 * Br:3 * Br + 16]
            toks = vals[3 * Br + 16:]
            # the round's tree as built on the device (adaptive rounds may be smaller)
            n_tree = plan_dev[10] if nh > 0 else 1
            topk_round = plan_dev[2:2 + plan_dev[1]] if nh > 0 else []
            stats["total_verify_rounds"] += 1
            active_batch_sum += n_active
            tree_node_sum += n_tree
            tree_plan_last = {"B_cur": n_active, "node_budget_per_seq": plan.node_budget_per_seq,
                              "active_heads": plan.active_heads, "topk_by_depth": list(topk_round),
                              "actual_nodes": n_tree, "proposal_mode": "chain" if rcfg.chain else "medusa"}
            # what the next round's shape depends on now; the rest after its launch
            pend_before = [pending_host[r] for r in act_rows]
            for i, r in enumerate(act_rows):
                row_len_host[r] += acc_len[i]
                if fin[i]:
                    active_host[r] = False
                pending_host[r] = pend[i]
            deferred = (act_rows, acc_len, toks, dcap, n_tree, pend_before)
        if deferred is not None:
            account(deferred)
        total_time = time.time() - total_start
        rounds = max(stats["total_verify_rounds"], 1)
        decoded = max(stats["total_decoded_token_num"], 1)
        proposed = max(stats["total_proposed_medusa_tokens"], 1)
        avg_accept = stats["total_acc_length"] / decoded
        total_tokens = sum(len(g) for g in generated)
        return {
            "generated_token_ids": generated,
            "max_sequence_length": max((len(g) for g in generated), default=0),
            **stats,
            "average_accept_length": float(avg_accept),
            "accepted_tokens_per_medusa_step": float(avg_accept),
            "total_accepted_draft_tokens": stats["total_accepted_medusa_tokens"],
            "total_proposed_draft_tokens": stats["total_proposed_medusa_tokens"],
            "correction_token_rate": stats["total_correction_tokens"] / decoded,
            "draft_acceptance_rate": stats["total_accepted_medusa_tokens"] / proposed,
            "medusa_acceptance_rate": stats["total_accepted_medusa_tokens"] / proposed,
            "average_active_batch_size": active_batch_sum / rounds,
            "average_tree_nodes_per_seq": tree_node_sum / rounds,
            "accept_length_histogram": accept_hist,
            "medusa_accept_by_depth": accept_by_depth,
            "last_tree_plan": tree_plan_last,
            "cache_update_mode": cfg.cache_update_mode,
            "kv_extraction_success_count": stats["total_verify_rounds"],
            "kv_extraction_fallback_count": 0,
            "oom_count": 0,
            "total_time_cost": total_time,
            "prefill_time_cost": prefill_time,
            "tree_verify_time_cost": verify_time,
            "target_time_cost": prefill_time + verify_time,
            "tokens_per_sec_generation": total_tokens / max(total_time, 1e-9),
            "reflex_metrics": {"enabled": False},
        }

#!/usr/bin/env python
"""Accepted tokens/sec of the MEDUSA tree-verify round on B200.

Workload (the benchmark's config 2): Qwen2.5-1.5B-shaped random-init policy
(bf16, 28 layers, hidden 1536, 12/2 heads, head_dim 128, vocab 151936),
3 tied MEDUSA heads, 64 rollouts per GPU (8 prompts x 8 samples), 1024-token
uniform-random prefixes, concurrency-aware trees (cpeak_nodes 1024, at most
16 nodes -> plan [4, 2], 13 nodes, 2 active heads), temperature 1.0.

A step is one verify round over the rows: proposal GEMM + root sampling +
candidate top-k, tree build, 28-layer verify forward with tree attention,
internal-node lm_head, exact_target acceptance + extract_path compaction,
replayed from a CUDA graph.  `value` = accepted tokens of all ranks / the
slowest rank's device time (CUDA events) over `--steps` steps.  Inputs are
larger than L2 (3.1 GB of weights and a 1.9 GB KV cache are read per step).
`e2e` runs config 2's rollout through the public API: generate() on 8
prompts of 256 uniform-random tokens (x8 samples) until every row holds 1024
tokens, prompts copied from pinned host memory and tokens read back each
round, timed on the host clock.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU)
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "ss-grpo_b200"))
sys.path.insert(0, str(REPO))

METRIC = "accepted tokens/sec per box at 1/2/4/8 B200; tree-attn HBM GB/s vs peak"
UNIT = "accepted tokens/s"

# The benchmark's GPU configurations, per GPU (configs 3 and 4 are quoted
# for 8 GPUs: 128 and 256 rollouts sharded by sequence, 16 and 32 per GPU).
RUNS = {
    2: dict(workload="config 2: Qwen2.5-1.5B-shaped MEDUSA tree-verify round", rows=64, prefix=1024, heads=3,
            cpeak=1024, max_nodes=16, depth=4, topk=(4, 3, 2), adaptive=False, adaptive_min=(1, 1, 1),
            chain=False, e2e_prompt=256, e2e_len=1024),
    3: dict(workload="config 3: Qwen2.5-7B-shaped MEDUSA tree-verify round (adaptive top-k 2..8, 32 nodes)",
            rows=16, prefix=2048, heads=4, cpeak=1024, max_nodes=32, depth=5, topk=(8, 8, 8, 8), adaptive=True,
            adaptive_min=(2, 2, 2, 2), chain=False, e2e_prompt=2048, e2e_len=2048 + 64),
    4: dict(workload="config 4: Llama-3.1-8B-shaped chain-proposal tree-verify round (up to 64 nodes)",
            rows=32, prefix=4096, heads=3, cpeak=2048, max_nodes=64, depth=4, topk=(4, 4, 4), adaptive=False,
            adaptive_min=(1, 1, 1), chain=True, e2e_prompt=4096, e2e_len=4096 + 64),
}
WORKLOAD = RUNS[2]["workload"]
CONFIG_LAYERS = {2: 28, 3: 28, 4: 32}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=sorted(RUNS), default=2,
                    help="benchmark configuration (2: the headline; 3, 4: the 7B / 8B-shaped per-GPU shards)")
    ap.add_argument("--sweep", choices=["attention", "lm-head"], default=None,
                    help="attention: config 5, tree attention + extract_path over prefix length x nodes x batch; "
                         "lm-head: config 2's proposal lm_head, the reference's separate leaf recompute against "
                         "the one fused projection")
    ap.add_argument("--sweep-max-gb", type=float, default=80.0,
                    help="skip sweep points whose K/V cache exceeds this many GB")
    ap.add_argument("--sweep-only", default=None,
                    help="run only these sweep points, as L:N:B[,L:N:B...] (profiling a single point)")
    ap.add_argument("--rows", type=int, default=None, help="rollouts per GPU (prompts x 8; default: the config's)")
    ap.add_argument("--prefix", type=int, default=None, help="prefix tokens (default: the config's)")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (profiling only)")
    ap.add_argument("--e2e-calls", type=int, default=2)
    ap.add_argument("--e2e-prompt", type=int, default=None,
                    help="e2e prompt tokens (config 2: 256-token prompts whose KV grows to --e2e-len by decoding)")
    ap.add_argument("--e2e-len", type=int, default=None, help="e2e max_length: prompt + generated tokens per row")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--attn-splits", type=int, default=0)
    ap.add_argument("--lm-head", choices=["fused", "separate"], default="separate",
                    help="proposal lm_head: tcgen05 GEMM with fused top-k, or cuBLAS + row top-k")
    ap.add_argument("--dense", choices=["auto", "native", "cublas"], default="auto",
                    help="verify projections + internal lm_head: per shape the faster of fg_linear and cuBLAS, "
                         "fg_linear (tcgen05) always, or cuBLAS")
    args = ap.parse_args()
    run = RUNS[args.config]
    for k in ("rows", "prefix", "e2e_prompt", "e2e_len"):
        if getattr(args, k) is None:
            setattr(args, k, run[k])
    return args


def measured_peaks() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic() -> float | None:
    """dram read+write bytes per tree-attention launch from the committed ncu summary."""
    p = REPO / "profiles" / "tree_attention_config2.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["dram_bytes_per_launch_full_model"])
        except (KeyError, ValueError):
            return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons, sampled every 20 ms from before
    the warm-up until after the timed region; `summary` keeps the samples
    whose timestamps fall inside the timed window (marked with `mark`)."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        import tempfile

        self.gpu = gpu_index
        self.proc = None
        self.window = None
        fd, name = tempfile.mkstemp(prefix=f"fg_clocks_gpu{gpu_index}_", suffix=".csv")
        os.close(fd)
        self.path = Path(name)

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def mark(self, t0: float, t1: float):
        """Wall-clock bounds (time.time()) of the timed region."""
        self.window = (t0, t1)

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        from datetime import datetime

        samples = []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                samples.append((ts, float(parts[2]), float(parts[3]),
                                {n for n, v in zip(names, parts[6:10]) if v.lower() == "active"}))
            except ValueError:
                continue
        inside = samples
        if self.window is not None:
            t0, t1 = self.window
            inside = [x for x in samples if t0 <= x[0] <= t1]
            if not inside and samples:  # region shorter than the sampling period: nearest sample
                mid = 0.5 * (t0 + t1)
                inside = [min(samples, key=lambda x: abs(x[0] - mid))]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(x[1] for x in inside), "sm_max_mhz": inside[-1][2],
                "reasons": sorted(set().union(*(x[3] for x in inside))), "samples": len(inside)}


# --------------------------------------------------------------- workload
def plan_for(cfg_id: int, rows: int):
    """The configuration's tree plan for `rows` rollouts on one GPU (host planner)."""
    from flashgrpo_b200.decoding.medusa_tree import dense_topology, plan_tree

    r = RUNS[cfg_id]
    plan = plan_tree(active_batch_size=rows, num_medusa_heads=r["heads"], tree_mode="concurrency_aware",
                     cpeak_nodes=r["cpeak"], min_tree_nodes_per_seq=1, max_tree_nodes_per_seq=r["max_nodes"],
                     max_tree_depth=r["depth"], fixed_tree_topk_by_depth=list(r["topk"]),
                     adaptive_tree_enabled=r["adaptive"], adaptive_min_topk_by_depth=list(r["adaptive_min"]))
    return plan, len(dense_topology(plan)[0])


def workload_config(cfg_id: int, rows: int, prefix: int, layers: int, world: int) -> dict:
    """The `config` object both arms print: the workload, not the engine."""
    r = RUNS[cfg_id]
    plan, n_nodes = plan_for(cfg_id, rows)
    out = {"workload": r["workload"], "rollouts_per_gpu": rows, "prompts_per_gpu": max(1, rows // 8),
           "samples_per_prompt": 8, "prefix_tokens": prefix, "tree": list(plan.topk_by_depth),
           "tree_nodes": n_nodes, "layers": layers, "medusa_heads": r["heads"], "active_heads": plan.active_heads,
           "temperature": 1.0, "top_p": 1.0, "parallelism": f"dp{world} (rollouts sharded by prompt group)"}
    if r["adaptive"]:
        out["adaptive_topk"] = [min(r["adaptive_min"]), max(r["topk"])]
    if r["chain"]:
        out["proposal_mode"] = "chain"
    return out


def decoder_for(cfg_id: int, device, layers=None, attn_splits=0, lm_head="separate", dense="auto"):
    import torch

    from flashgrpo_b200.decoding.flash_medusa_decoder import FlashMedusaConfig, FlashMedusaDecoder
    from flashgrpo_b200.utils import synthetic

    r = RUNS[cfg_id]
    over = {} if layers is None else {"layers": layers}
    model = synthetic.build_model(cfg_id, device=device, attn_implementation="sdpa", **over)
    heads = synthetic.medusa_head_tensors(cfg_id, device=device, chain=r["chain"])

    class Tok:
        pad_token_id = 0
        eos_token_id = 1

    cfg = FlashMedusaConfig(num_medusa_heads=r["heads"], tree_mode="concurrency_aware", cpeak_nodes=r["cpeak"],
                            max_tree_nodes_per_seq=r["max_nodes"], max_tree_depth=r["depth"],
                            fixed_tree_topk_by_depth=tuple(r["topk"]), adaptive_tree_enabled=r["adaptive"],
                            adaptive_min_topk_by_depth=tuple(r["adaptive_min"]),
                            proposal_mode="chain" if r["chain"] else "medusa",
                            temperature=1.0, top_p=1.0, sampling_seed=1234, attention_splits=attn_splits,
                            lm_head_kernel=lm_head, dense_kernel=dense)
    torch.cuda.synchronize()
    return FlashMedusaDecoder(model, heads, Tok(), cfg)


def attention_back_to_back(eng, st, rb, rcfg, reps: int = 2) -> float:
    """Average device time (ms) of the round's tree-attention call, launched
    back to back over every layer's KV cache with CUDA events around the
    whole sweep: the kernel's own duration, without the graph's event nodes
    and launch gaps that bracket a single in-round launch.  Each layer's cache
    (81 MB in config 2) was last read n_layers - 1 launches earlier, so no
    launch finds its K/V in L2."""
    import torch

    from flashgrpo_b200 import ops

    ws = eng._attn_workspace(rb, st, rcfg.attn_splits)

    def sweep():
        for l in range(eng.spec.n_layers):
            ops.tree_attention(rb.q, st.k[l], st.v[l], st.row_len, rb.tree["anc"], scale=eng.scale, out=rb.attn,
                               workspace=ws, num_splits=rcfg.attn_splits, max_kv_len=st.capacity,
                               kv=st.kv_layers[l])

    sweep()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        sweep()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / (reps * eng.spec.n_layers)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from flashgrpo_b200 import _native
    from flashgrpo_b200.engine import shard
    from flashgrpo_b200.engine.verify import DecodeState  # noqa: F401
    from flashgrpo_b200.utils import synthetic

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    torch.manual_seed(0)
    run = RUNS[args.config]
    dec = decoder_for(args.config, device, args.layers, args.attn_splits, args.lm_head, args.dense)
    eng = dec.engine
    spec = eng.spec
    # the global batch is world x prompts prompt groups; this rank owns a
    # contiguous range of whole groups (8 samples of a prompt stay together)
    prompts = max(1, args.rows // 8)
    my_prompts = shard.prompt_shard(prompts * world, world, rank)
    ids_all, mask_all = synthetic.random_prompts(prompts * world, args.prefix, spec.vocab, seed=100)
    ids, mask = ids_all[my_prompts.start:my_prompts.stop], mask_all[my_prompts.start:my_prompts.stop]
    rows = len(my_prompts) * 8
    # every rank's rollout count, from the shard plan (sizes of the one all-gather)
    counts = [len(shard.prompt_shard(prompts * world, world, r)) * 8 for r in range(world)]
    W, K = max(args.warmup, 3), max(args.steps, 1)
    # a round retires at most `depth` tokens per row and writes its tree after them
    capacity = args.prefix + run["depth"] * (W + K + 8) + run["max_nodes"] + 8
    n_heads = dec.max_heads()
    rcfg = dec.round_config(max_length=1 << 30)
    with torch.inference_mode():
        st = eng.prefill(ids, mask, repeats=8, capacity=capacity, n_heads=n_heads)
        plan = dec._plan(rows)
        nh = min(n_heads, plan.active_heads)
        plan.topk_by_depth, plan.active_heads = plan.topk_by_depth[:nh], nh
        rb = eng.buffers(rows, plan, nh, nh + 2, adaptive=run["adaptive"] and nh > 0)
        params = dec._params(rows)
        # two warm-up rounds eagerly: the first meets the lazy cuBLAS /
        # allocator state and tunes the projection tilings, the second counts
        # the library's kernel launches of one steady-state round
        eng.run_round(st, rb, params, rcfg)
        torch.cuda.synchronize()
        before = _native.launches
        eng.run_round(st, rb, params, rcfg)
        launches_per_step = _native.launches - before
        torch.cuda.synchronize()
        # G graphs in rotation, each with its own per-layer attention events
        G = min(4, K)
        # live timing of the tree attention of layer 0 in every timed step; the
        # other layers carry no events, so their attention overlaps the tail
        # of the RoPE/KV write before it (programmatic launch)
        events = [[(torch.cuda.Event(enable_timing=True, external=True),
                    torch.cuda.Event(enable_timing=True, external=True))] + [None] * (spec.n_layers - 1)
                  for _ in range(G)]
        graphs = []
        pool = None
        for gi in range(G):
            g = eng.graph_round(st, rb, params, rcfg, pool=pool, attn_events=events[gi])
            pool = g.pool()
            graphs.append(g)
        clocks = ClockSampler(local_rank).__enter__()
        for i in range(W - 1):
            graphs[i % G].replay()
        torch.cuda.synchronize()
        acc0 = int(rb.acc_sum.item())
        len0 = st.row_len.float().mean().item()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        w0 = time.time()
        # an NVTX range around the timed steps, so a profiler can keep to them
        torch.cuda.nvtx.range_push("fg_timed_steps")
        t_start.record()
        for i in range(K):
            graphs[i % G].replay()
        t_end.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        clocks.mark(w0, time.time())
        clocks.__exit__(None, None, None)
        if world > 1:
            dist.barrier()
        ms = t_start.elapsed_time(t_end)
        accepted = int(rb.acc_sum.item()) - acc0
        len1 = st.row_len.float().mean().item()
        # the last G steps' layer-0 attention launches
        attn_ms = [events[(K - 1 - j) % G][0][0].elapsed_time(events[(K - 1 - j) % G][0][1]) for j in range(G)]
        err = _native.read_device_error(clear=True)
        if err:
            raise RuntimeError(f"device error word {err} after the timed region")
        # the same attention call back to back over the 28 layers' caches
        attn_b2b_ms = attention_back_to_back(eng, st, rb, rcfg)
        rollout_len = (st.row_len - args.prefix).clone()
        del graphs
        # ---- roofline of the tree-attention kernel (K3)
        N_ = rb.N
        L_avg = 0.5 * (len0 + len1)
        hq, hkv, D = spec.n_q_heads, spec.n_kv_heads, spec.head_dim
        attn_bytes = rows * hkv * (L_avg + N_) * D * 2 * 2 + rows * N_ * hq * D * 2 * 2
        attn_avg_ms = statistics.mean(attn_ms)
        # K/V of every row's prefix + tree and the Q/out rows, at the lengths
        # the back-to-back sweep saw (after the timed steps)
        attn_bytes_b2b = rows * hkv * (len1 + N_) * D * 2 * 2 + rows * N_ * hq * D * 2 * 2
        achieved = attn_bytes_b2b / (attn_b2b_ms * 1e-3) / 1e9
        # QK^T and PV over every prefix + tree slot: N x G query rows per KV head
        attn_flops_b2b = 4.0 * rows * hq * N_ * (len1 + N_) * D
        tflops_peak, _ = measured_tensor_peak()
        peak, peak_kind = measured_peaks()
        traffic = profile_traffic() if args.config == 2 and args.rows == 64 and args.prefix == 1024 else None
        # ---- end-to-end through the public generate() API (prompts H2D, tokens D2H)
        e2e = None
        if not args.no_e2e and args.e2e_calls > 0:
            # the configuration's rollout through the public generate() call
            # (config 2: 256-token prompts decoded until the rows hold 1024 tokens)
            e_all, m_all = synthetic.random_prompts(prompts * world, args.e2e_prompt, spec.vocab, seed=101)
            e_ids = e_all[my_prompts.start:my_prompts.stop].pin_memory()
            e_mask = m_all[my_prompts.start:my_prompts.stop].pin_memory()
            # warm-up calls with the timed calls' arguments (W of them, at most
            # 3): the same decode state and round configuration, so every timed
            # round replays a captured graph, and the HF prefill has settled
            # (its first calls take 1.9 / 0.2 / 0.1 s, then 0.017 s)
            for _ in range(min(W, 3)):
                dec.generate(e_ids, e_mask, repeated_generate_nums=8, max_length=args.e2e_len)
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            t0 = time.perf_counter()
            tok, rounds_total, pre_s, ver_s = 0, 0, 0.0, 0.0
            for _ in range(args.e2e_calls):
                res = dec.generate(e_ids, e_mask, repeated_generate_nums=8, max_length=args.e2e_len)
                tok += res["total_acc_length"]
                rounds_total += res["total_verify_rounds"]
                pre_s += res["prefill_time_cost"]
                ver_s += res["total_time_cost"] - res["prefill_time_cost"]
            torch.cuda.synchronize()
            e_local_s = time.perf_counter() - t0
            dcap = plan.active_heads + 2
            e2e = {"unit": UNIT,
                   "h2d_bytes_per_step": int(e_ids.numel() * 8 + e_mask.numel() * 8),
                   "d2h_bytes_per_step": int(rounds_total / args.e2e_calls * rows * (3 + dcap) * 4),
                   "step": f"one generate() call: {prompts} prompts x {args.e2e_prompt} tokens prefilled, x8 samples, "
                           f"decoded to max_length {args.e2e_len}",
                   "calls": args.e2e_calls, "prefill_s_per_call": pre_s / args.e2e_calls,
                   "verify_rounds_s_per_call": ver_s / args.e2e_calls, "rounds_per_call": rounds_total / args.e2e_calls}
        # the one collective: a single all-gather of every rank's per-rollout
        # generated lengths (the GRPO group statistics), carrying each rank's
        # device time, accepted tokens and end-to-end seconds / tokens
        extras = [ms, accepted, e_local_s if e2e else 0.0, tok if e2e else 0]
        lengths_all, per_rank = shard.gather_rollouts(rollout_len, counts, extras=extras)
        ms_max = float(per_rank[:, 0].max())
        accepted_all = int(per_rank[:, 1].sum())
        if e2e is not None:
            e_s = float(per_rank[:, 2].max())
            e2e["value"] = float(per_rank[:, 3].sum()) / e_s
            e2e["per_rank"] = [float(t / x) for x, t in zip(per_rank[:, 2].tolist(), per_rank[:, 3].tolist())]
    weight_gb = sum(p.numel() * p.element_size() for p in dec.target_model.parameters()) / 1e9
    kv_gb = 2 * spec.n_layers * rows * spec.n_kv_heads * (len1 + rb.N) * spec.head_dim * 2 / 1e9
    result = {
        "metric": METRIC, "value": accepted_all / (ms_max * 1e-3), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic: random-init weights N(0,0.02), uniform-random prompt ids",
        "config": workload_config(args.config, rows, args.prefix, spec.n_layers, world),
        "engine": {"lm_head": args.lm_head, "dense": args.dense,
                   "dense_shapes": {f"{k[0]}x{k[1]}x{k[2]}/{['store', 'resid', 'swiglu'][k[3]]}": v
                                    for k, v in eng.tile_report.items()},
                   "l2": f"inputs larger than L2: {weight_gb:.1f} GB of weights and a {kv_gb:.1f} GB KV cache "
                         "read every step",
                   "graphs": "each step replays a captured CUDA graph of the round"},
        "accepted_tokens": accepted_all, "average_accept_length": accepted_all / (K * rows * world),
        "rollouts_gathered": int(lengths_all.numel()),
        "gpu_launches": launches_per_step * K,
        "roofline": {"kernel": "fg_tree_attention (fg::tc::attn_tc_kernel, tcgen05)", "bound": "hbm",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback", "traffic": traffic,
                     "algorithmic_bytes_per_launch": attn_bytes_b2b, "avg_launch_ms": attn_b2b_ms,
                     "flops_per_launch": attn_flops_b2b,
                     "intensity_flop_per_byte": attn_flops_b2b / attn_bytes_b2b,
                     "ridge_flop_per_byte": tflops_peak * 1e12 / (peak * 1e9),
                     "tensor_frac": attn_flops_b2b / (attn_b2b_ms * 1e-3) / 1e12 / tflops_peak,
                     "launches_timed": 2 * spec.n_layers,
                     "timing": f"CUDA events around {2 * spec.n_layers} back-to-back launches of the round's "
                               f"attention call over the {spec.n_layers} layers' KV caches (no L2 reuse), after the "
                               "timed steps",
                     "in_round": {"avg_launch_ms": attn_avg_ms, "algorithmic_bytes_per_launch": attn_bytes,
                                  "achieved": attn_bytes / (attn_avg_ms * 1e-3) / 1e9, "launches_timed": len(attn_ms),
                                  "timing": "CUDA events around the layer-0 attention node of the last replayed "
                                            "round graphs (includes the graph's event-node and launch gaps; the "
                                            "events also keep that launch from overlapping the RoPE/KV write)"}},
        "clocks": clocks.summary(),
    }
    if e2e is not None:
        result["e2e"] = e2e
    return result


# ---------------------------------------------------------- config 5 sweep
SWEEP_L = (1024, 4096, 16384, 32768)
SWEEP_N = (8, 16, 64, 128)
SWEEP_B = (1, 32, 128, 512)


def measured_tensor_peak() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def random_tree(n: int, g, max_depth: int = 4) -> list[int]:
    """Seeded parent array of a dense tree in topological order: node j's
    parent is drawn uniformly from the earlier nodes less than `max_depth`
    deep, so root-to-leaf paths stay within the accepted-path limit."""
    import torch

    parents, depth = [-1], [0]
    for j in range(1, n):
        cand = [i for i in range(j) if depth[i] < max_depth]
        p = cand[int(torch.randint(0, len(cand), (1,), generator=g))]
        parents.append(p)
        depth.append(depth[p] + 1)
    return parents


def graph_time(launches, min_ms: float = 20.0) -> tuple[float, int]:
    """Average device time (ms) of one call in `launches`: the calls are
    captured once into a CUDA graph (so the host's launch rate does not
    limit small ones) and the graph is replayed until >= min_ms of device
    time, between CUDA events.  Returns (ms per call, calls timed)."""
    import math

    import torch

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for f in launches:
            f()
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    n = max(1, math.ceil(min_ms / max(e0.elapsed_time(e1), 1e-3)))
    e0.record()
    for _ in range(n):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (n * len(launches))
    del graph
    return ms, n * len(launches)


def run_sweep(args, local_rank: int) -> dict:
    """Config 5: fg_tree_attention and fg_extract_path alone, bf16, N(0, 1)
    K/V, GQA 32 q / 8 kv heads, head_dim 128, over prefix length x tree nodes
    x batch.  Each point rotates its launches over enough distinct K/V
    copies (>= 320 MB together, 2.5x L2) that no launch finds its K/V in L2;
    the largest points are single copies far larger than L2.  Time: CUDA
    events around CUDA-graph replays of the rotation, after 3 untimed
    launches."""
    import math

    import torch

    from flashgrpo_b200 import _native, ops
    from flashgrpo_b200.models.hf_tree_attention import ancestor_bits

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    hq, hkv, D = 32, 8, 128
    hbm, hbm_kind = measured_peaks()
    tf, tf_kind = measured_tensor_peak()
    ridge = tf * 1e12 / (hbm * 1e9)  # flop per byte
    slot = hkv * D * 2  # bytes of one K (or V) slot of one row
    cap_bytes = args.sweep_max_gb * 1e9
    grid = [(L, N, B) for L in SWEEP_L for N in SWEEP_N for B in SWEEP_B]
    if args.sweep_only:
        grid = [tuple(int(x) for x in pt.split(":")) for pt in args.sweep_only.split(",")]
        if any(len(pt) != 3 or min(pt) <= 0 or pt[1] > 128 for pt in grid):
            raise SystemExit("--sweep-only wants L:N:B points with N <= 128")
    kv_need = {pt: 2 * pt[2] * (pt[0] + pt[1]) * slot for pt in grid}
    runnable = [pt for pt in grid if kv_need[pt] <= cap_bytes]
    rot_bytes = 320e6
    pool_bytes = max(min(cap_bytes, max(kv_need[pt], rot_bytes * 1.05)) for pt in runnable)
    pool = torch.empty(int(pool_bytes // 2), dtype=torch.bfloat16, device=device)
    g = torch.Generator(device=device).manual_seed(5)
    pool.normal_(generator=g)
    gh = torch.Generator().manual_seed(7)
    scale = 1.0 / math.sqrt(D)
    points = []
    for (L, N, B) in grid:
        rec = {"L": L, "N": N, "B": B}
        if (L, N, B) not in runnable:
            rec["skipped"] = f"K/V cache {kv_need[(L, N, B)] / 1e9:.1f} GB above --sweep-max-gb"
            points.append(rec)
            continue
        cap = L + N
        per = B * hkv * cap * D  # elements of one K (or V) cache
        copies = max(1, min(256, math.ceil(rot_bytes / kv_need[(L, N, B)]), pool.numel() // (2 * per)))
        caches = []
        for c in range(copies):
            base = c * 2 * per
            k = pool[base:base + per].view(B, hkv, cap, D)
            v = pool[base + per:base + 2 * per].view(B, hkv, cap, D)
            caches.append((k, v, ops.kv_layer(k, v)))
        parents = random_tree(N, gh)
        anc = ancestor_bits(parents, device=device)
        q = torch.randn(copies, B, N, hq, D, device=device, dtype=torch.bfloat16, generator=g)
        out = torch.empty(B, N, hq, D, device=device, dtype=torch.bfloat16)
        kv_len = torch.full((B,), L, dtype=torch.int32, device=device)
        ws_bytes = ops.attention_workspace_bytes(B, N, hq, hkv, D, max_kv_len=cap)
        # split-K partials and the self-resetting merge counters start at zero
        ws = torch.zeros(max(ws_bytes, 16), dtype=torch.uint8, device=device)

        def launch(c):
            k, v, kv = caches[c]
            ops.tree_attention(q[c], k, v, kv_len, anc, scale=scale, out=out, workspace=ws, max_kv_len=cap, kv=kv)

        for i in range(3):
            launch(i % copies)
        torch.cuda.synchronize()
        ms, reps = graph_time([lambda c=c: launch(c) for c in range(copies)])
        kv_bytes = 2 * B * hkv * (L + N) * D * 2
        qo_bytes = 2 * B * N * hq * D * 2
        byts = kv_bytes + qo_bytes
        flops = 4.0 * B * hq * N * (L + N) * D
        t_roof = max(byts / (hbm * 1e9), flops / (tf * 1e12))
        # extract_path of a random root-to-leaf path per row (one layer)
        depth = [0] * N
        for j in range(1, N):
            depth[j] = depth[parents[j]] + 1
        leaves = [j for j in range(N) if j not in set(parents)]
        dcap = max(depth) + 1
        acc_nodes = torch.full((B, dcap), -1, dtype=torch.int32)
        acc_len = torch.empty(B, dtype=torch.int32)
        for b in range(B):
            j = leaves[int(torch.randint(0, len(leaves), (1,), generator=gh))]
            path = []
            while j >= 0:
                path.append(j)
                j = parents[j]
            path.reverse()
            acc_nodes[b, :len(path)] = torch.tensor(path, dtype=torch.int32)
            acc_len[b] = len(path)
        acc_nodes, acc_len = acc_nodes.to(device), acc_len.to(device)
        moved = int(sum((int(a) - 1) for a in acc_len.tolist())) * hkv * D * 2 * 2 * 2
        for c in range(min(copies, 3)):
            ops.extract_path([caches[c][0]], [caches[c][1]], kv_len, acc_nodes, acc_len)
        torch.cuda.synchronize()
        x_ms, _ = graph_time([lambda c=c: ops.extract_path([caches[c % copies][0]], [caches[c % copies][1]], kv_len,
                                                           acc_nodes, acc_len) for c in range(max(copies, 16))])
        err = _native.read_device_error(clear=True)
        if err:
            raise RuntimeError(f"device error word {err} at sweep point L={L} N={N} B={B}")
        rec.update({"intensity_flop_per_byte": flops / byts, "bound": "hbm" if flops / byts < ridge else "tensor",
                    "ms": ms, "GB_s": byts / (ms * 1e-3) / 1e9, "TFLOP_s": flops / (ms * 1e-3) / 1e12,
                    "hbm_frac": byts / (ms * 1e-3) / 1e9 / hbm, "tensor_frac": flops / (ms * 1e-3) / 1e12 / tf,
                    "frac": t_roof / (ms * 1e-3), "algorithmic_bytes": byts,
                    "splits": None if ws_bytes == 0 else "auto (>1)", "kv_copies": copies, "launches_timed": reps,
                    "extract_us": x_ms * 1e3, "extract_bytes": moved})
        points.append(rec)
        print(f"L={L:6d} N={N:4d} B={B:4d}  {ms * 1e3:10.1f} us  {rec['GB_s']:8.1f} GB/s  "
              f"{rec['TFLOP_s']:7.1f} TF/s  frac {rec['frac']:.3f} ({rec['bound']})  extract {x_ms * 1e3:.1f} us",
              file=sys.stderr, flush=True)
        del caches, q, out, ws, kv_len, anc
    return {"sweep": "config 5: isolated tree attention + extract_path (one layer), bf16, random N(0,1) K/V, "
                     "GQA 32 q / 8 kv heads, head_dim 128, seeded random dense trees (depth <= 4), a random "
                     "accepted root-to-leaf path per row",
            "peaks": {"hbm_gbs": hbm, "hbm_source": hbm_kind, "bf16_tflops": tf, "tensor_source": tf_kind,
                      "ridge_flop_per_byte": ridge},
            "bytes": "2*B*Hkv*(L+N)*D*2 (K and V of prefix + tree) + 2*B*N*Hq*D*2 (Q in, O out)",
            "flops": "4*B*Hq*N*(L+N)*D (QK^T and PV over every slot)",
            "l2": "launches rotate over distinct K/V and Q copies of >= 320 MB together (or one copy larger than L2)",
            "points": points}


def run_lmhead_sweep(args, local_rank: int) -> dict:
    """Config 2's vocabulary projections around a round boundary (H 1536,
    V 151,936, bf16, 64 rows, 2 active MEDUSA heads, top-4), timed alone
    with CUDA graphs over 3 rotating weight copies (1.4 GB, so every call
    streams its 467 MB of weights from HBM):
      reference  the leaf-logit recompute after acceptance
                 (flash_medusa_decoder.py:2836-2862: lm_head on the 64 last
                 accepted hidden states) and, next round, the heads' lm_head
                 on 128 rows + their top-k: two weight streams;
      fused      this repository's round: the last accepted hidden state is
                 gathered by K4 and projected in the next round's one GEMM
                 together with the head rows (M = 192) + the top-k of the
                 head rows: one weight stream;
      tcgen05    the same fused projection as fg_lm_head_topk (the top-k in
                 the GEMM epilogue)."""
    import torch

    from flashgrpo_b200 import ops

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    B, H, V, k, heads = 64, 1536, 151936, 4, 2
    g = torch.Generator(device=device).manual_seed(3)
    W = [torch.randn(V, H, device=device, generator=g).mul_(0.02).to(torch.bfloat16) for _ in range(3)]
    X = torch.randn((1 + heads) * B, H, device=device, generator=g).to(torch.bfloat16)
    logits = torch.empty((1 + heads) * B, V, device=device, dtype=torch.bfloat16)
    n_top = heads * B
    tk = (torch.empty((n_top, k), dtype=torch.int32, device=device), torch.empty((n_top, k), device=device),
          torch.empty(n_top, device=device), None)
    ws = torch.empty(max(ops.lm_head_topk_workspace_bytes(X.shape[0], V, B, k), 16) // 4 + 64, dtype=torch.int32,
                     device=device)

    def reference(i):
        w = W[i % 3]
        torch.mm(X[:B], w.t(), out=logits[:B])          # leaf recompute after acceptance
        torch.mm(X[B:], w.t(), out=logits[B:])          # next round: the heads' projection
        ops.row_topk(logits[B:], k, out=tk, with_lse=False)

    def fused(i):
        torch.mm(X, W[i % 3].t(), out=logits)
        ops.row_topk(logits[B:], k, out=tk, with_lse=False)

    def tcgen05(i):
        ops.lm_head_topk(X, W[i % 3], n_logit_rows=B, logits=logits, topk_row0=B, k=k, topk_out=tk, workspace=ws)

    peak, _ = measured_peaks()
    out = {"sweep": "config 2 proposal lm_head: the reference's separate leaf-logit recompute against one fused "
                    "projection (64 rows, 2 heads, H 1536, V 151,936, bf16, top-4)", "variants": {}}
    for name, fn, streams in (("reference", reference, 2), ("fused", fused, 1), ("tcgen05", tcgen05, 1)):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        ms, n = graph_time([lambda i=i: fn(i) for i in range(3)])
        wbytes = streams * V * H * 2
        out["variants"][name] = {"us": ms * 1e3, "weight_streams": streams,
                                 "weight_GB_s": wbytes / (ms * 1e-3) / 1e9, "hbm_frac": wbytes / (ms * 1e-3) / 1e9 / peak,
                                 "calls_timed": n}
        print(f"{name:10s} {ms * 1e3:8.1f} us  {streams} weight stream(s)", file=sys.stderr, flush=True)
    return out


# ------------------------------------------------------------- CPU oracle
def cpu_oracle_round_rate(warm_rounds: int, timed_rounds: int, rows: int = 64, prefix: int = 1024, cfg_id: int = 2):
    """The oracle's restatement of the reference generate loop on the host
    cores, on the configuration's own shape (fp32): `rows` rollouts (rows / 8
    prompts x 8 samples) of `prefix`-token uniform-random prompts, the same
    tree plan (config 2: cpeak 1024, at most 16 nodes), HF eager attention
    with the dense tree mask.  The prefill is not timed; `timed_rounds` verify
    rounds after `warm_rounds` are."""
    import torch

    from oracle import reference_path as rp
    from flashgrpo_b200.utils import synthetic

    torch.set_num_threads(os.cpu_count() or 1)
    r = RUNS[cfg_id]
    model = synthetic.build_model(cfg_id, device="cpu", dtype=torch.float32, attn_implementation="eager",
                                  fast_host_init=True)
    st = synthetic.medusa_head_tensors(cfg_id, dtype=torch.float32, chain=r["chain"])

    def synthetic_prefill(model, ids, mask, pos, cache):
        """The prefix's K/V and hidden states at their shapes (N(0, 1)): the
        timed verify rounds read them like a prefilled cache, without the
        minutes a CPU prefill of 8 x 1024 tokens takes."""
        conf = model.config
        P, S = ids.shape
        hkv, D = conf.num_key_value_heads, conf.head_dim
        g = torch.Generator().manual_seed(5)
        for layer in range(conf.num_hidden_layers):
            k = torch.randn(P, hkv, S, D, generator=g)
            v = torch.randn(P, hkv, S, D, generator=g)
            cache.update(k, v, layer)
        return torch.randn(P, S, conf.hidden_size, generator=g), cache

    heads = [{"norm_w": st[f"heads.{i}.norm.weight"], "norm_b": st[f"heads.{i}.norm.bias"],
              "fc_w": st[f"heads.{i}.fc.weight"], "fc_b": st[f"heads.{i}.fc.bias"]} for i in range(r["heads"])]
    prompts = max(1, rows // 8)
    ids, mask = synthetic.random_prompts(prompts, prefix, synthetic.CONFIGS[cfg_id]["vocab"], seed=100)
    chain_cell = {k[len("chain_cell."):]: v for k, v in st.items() if k.startswith("chain_cell.")} or None
    cfg = rp.OracleConfig(num_medusa_heads=r["heads"], tree_mode="concurrency_aware", cpeak_nodes=r["cpeak"],
                          max_tree_nodes_per_seq=r["max_nodes"], max_tree_depth=r["depth"],
                          fixed_tree_topk_by_depth=tuple(r["topk"]), top_p=1.0,
                          adaptive_tree_enabled=r["adaptive"], adaptive_min_topk_by_depth=tuple(r["adaptive_min"]),
                          proposal_mode="chain" if r["chain"] else "medusa", chain_cell=chain_cell)
    t0 = time.perf_counter()
    res = rp.generate(model, heads, ids, mask, cfg, rp.SeqRoundSampler(1234), repeats=8,
                      max_length=prefix + warm_rounds + timed_rounds + 2, prefill_fn=synthetic_prefill)
    wall = time.perf_counter() - t0
    times = res["round_times"][warm_rounds:warm_rounds + timed_rounds]
    sec = sum(t for t, _ in times)
    tok = sum(n for _, n in times)
    return {"value": tok / sec, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(times)} verify rounds (after {warm_rounds} untimed) of config {cfg_id}'s full shape: "
                      f"{rows} rollouts ({prompts} prompts x 8 samples) with {prefix}-token prefixes, "
                      f"{synthetic.CONFIGS[cfg_id]['layers']} layers, "
                      "fp32 on the host; oracle/reference_path.py restatement of the reference generate loop "
                      "with HF eager attention and the dense tree mask; the prefix K/V are synthesized at their "
                      "shapes instead of a CPU prefill, which no arm times",
            "seconds": sec, "prefill_s": res["prefill_time"], "wall_s": wall}


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return 0
        # config 2's shape on the host, a bounded number of rounds: each
        # round of 64 rollouts is seconds of fp32 CPU work
        W, K = min(max(args.warmup, 3), 3), min(max(args.steps, 1), 8)
        base = cpu_oracle_round_rate(W, K, rows=args.rows, prefix=args.prefix, cfg_id=args.config)
        line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": args.gpus,
                "steps": K, "warmup": W, "ms_per_step": 1e3 * base["seconds"] / K, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic: random-init weights N(0,0.02), uniform-random prompt ids",
                "config": workload_config(args.config, args.rows, args.prefix, CONFIG_LAYERS[args.config], args.gpus),
                "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0
    if args.sweep is not None:
        if rank == 0:
            fn = run_sweep if args.sweep == "attention" else run_lmhead_sweep
            print(json.dumps(fn(args, local_rank)), flush=True)
        return 0
    import torch
    import torch.distributed as dist

    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local_rank))
    try:
        result = run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.barrier()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_oracle_round_rate(1, 3 if args.config == 2 else 2, rows=args.rows,
                                                           prefix=args.prefix, cfg_id=args.config)
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

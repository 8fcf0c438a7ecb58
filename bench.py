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
larger than L2 (3.1 GB of weights and a 3.7 GB KV cache are read per step).
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
WORKLOAD = "config 2: Qwen2.5-1.5B-shaped MEDUSA tree-verify round"


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--rows", type=int, default=64, help="rollouts per GPU (prompts x 8)")
    ap.add_argument("--prefix", type=int, default=1024)
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (profiling only)")
    ap.add_argument("--e2e-calls", type=int, default=2)
    ap.add_argument("--e2e-prompt", type=int, default=256,
                    help="e2e prompt tokens (config 2: 256-token prompts whose KV grows to --e2e-len by decoding)")
    ap.add_argument("--e2e-len", type=int, default=1024, help="e2e max_length: prompt + generated tokens per row")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--attn-splits", type=int, default=0)
    ap.add_argument("--lm-head", choices=["fused", "separate"], default="separate",
                    help="proposal lm_head: tcgen05 GEMM with fused top-k, or cuBLAS + row top-k")
    ap.add_argument("--dense", choices=["auto", "native", "cublas"], default="auto",
                    help="verify projections + internal lm_head: per shape the faster of fg_linear and cuBLAS, "
                         "fg_linear (tcgen05) always, or cuBLAS")
    return ap.parse_args()


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
def config2_plan(rows: int):
    """The config-2 tree plan for `rows` rollouts on one GPU (host planner)."""
    from flashgrpo_b200.decoding.medusa_tree import dense_topology, plan_tree

    plan = plan_tree(active_batch_size=rows, num_medusa_heads=3, tree_mode="concurrency_aware", cpeak_nodes=1024,
                     min_tree_nodes_per_seq=1, max_tree_nodes_per_seq=16, max_tree_depth=4,
                     fixed_tree_topk_by_depth=[4, 3, 2])
    return plan, len(dense_topology(plan)[0])


def workload_config(rows: int, prefix: int, layers: int, world: int) -> dict:
    """The `config` object both arms print: the workload, not the engine."""
    plan, n_nodes = config2_plan(rows)
    return {"workload": WORKLOAD, "rollouts_per_gpu": rows, "prompts_per_gpu": max(1, rows // 8),
            "samples_per_prompt": 8, "prefix_tokens": prefix, "tree": list(plan.topk_by_depth),
            "tree_nodes": n_nodes, "layers": layers, "medusa_heads": 3, "active_heads": plan.active_heads,
            "temperature": 1.0, "top_p": 1.0, "parallelism": f"dp{world} (rollouts sharded by prompt group)"}


def config2_decoder(device, layers=None, attn_splits=0, lm_head="separate", dense="auto"):
    import torch

    from flashgrpo_b200.decoding.flash_medusa_decoder import FlashMedusaConfig, FlashMedusaDecoder
    from flashgrpo_b200.utils import synthetic

    over = {} if layers is None else {"layers": layers}
    model = synthetic.build_model(2, device=device, attn_implementation="sdpa", **over)
    heads = synthetic.medusa_head_tensors(2, device=device)

    class Tok:
        pad_token_id = 0
        eos_token_id = 1

    cfg = FlashMedusaConfig(num_medusa_heads=3, tree_mode="concurrency_aware", cpeak_nodes=1024,
                            max_tree_nodes_per_seq=16, max_tree_depth=4, fixed_tree_topk_by_depth=(4, 3, 2),
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
    dec = config2_decoder(device, args.layers, args.attn_splits, args.lm_head, args.dense)
    eng = dec.engine
    spec = eng.spec
    # the global batch is world x prompts prompt groups; this rank owns a
    # contiguous range of whole groups (8 samples of a prompt stay together)
    prompts = max(1, args.rows // 8)
    my_prompts = shard.prompt_shard(prompts * world, world, rank)
    ids_all, mask_all = synthetic.random_prompts(prompts * world, args.prefix, spec.vocab, seed=100)
    ids, mask = ids_all[my_prompts.start:my_prompts.stop], mask_all[my_prompts.start:my_prompts.stop]
    rows = len(my_prompts) * 8
    W, K = max(args.warmup, 3), max(args.steps, 1)
    capacity = args.prefix + 3 * (W + K + 8) + 32
    n_heads = dec.max_heads()
    rcfg = dec.round_config(max_length=1 << 30)
    with torch.inference_mode():
        st = eng.prefill(ids, mask, repeats=8, capacity=capacity, n_heads=n_heads)
        plan = dec._plan(rows)
        rb = eng.buffers(rows, plan, plan.active_heads, plan.active_heads + 2)
        params = dec._params(rows)
        # warm-up round 1 eagerly (lazy cuBLAS / allocator state), counting our launches
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
        t_start.record()
        for i in range(K):
            graphs[i % G].replay()
        t_end.record()
        torch.cuda.synchronize()
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
        # the one collective: every rank's per-rollout generated lengths (for
        # the GRPO group statistics), then totals and the slowest clock
        rollout_len = (st.row_len - args.prefix).clone()
        lengths_all = shard.gather_rollout_values(rollout_len)
        ms_max = shard.reduce_scalar(ms, "max", device)
        accepted_all = int(shard.reduce_scalar(accepted, "sum", device))
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
        peak, peak_kind = measured_peaks()
        traffic = profile_traffic()
        # ---- end-to-end through the public generate() API (prompts H2D, tokens D2H)
        e2e = None
        if not args.no_e2e and args.e2e_calls > 0:
            # config 2's rollout: 256-token prompts decoded until the rows hold
            # 1024 tokens, through the public generate() call
            e_all, m_all = synthetic.random_prompts(prompts * world, args.e2e_prompt, spec.vocab, seed=101)
            e_ids = e_all[my_prompts.start:my_prompts.stop].pin_memory()
            e_mask = m_all[my_prompts.start:my_prompts.stop].pin_memory()
            # warm-up with the timed calls' arguments: the same decode state and
            # round configuration, so every timed round replays a captured graph
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
            e_s = shard.reduce_scalar(time.perf_counter() - t0, "max", device)
            tok = int(shard.reduce_scalar(tok, "sum", device))
            dcap = plan.active_heads + 2
            e2e = {"value": tok / e_s, "unit": UNIT,
                   "h2d_bytes_per_step": int(e_ids.numel() * 8 + e_mask.numel() * 8),
                   "d2h_bytes_per_step": int(rounds_total / args.e2e_calls * rows * (3 + dcap) * 4),
                   "step": f"one generate() call: {prompts} prompts x {args.e2e_prompt} tokens prefilled, x8 samples, "
                           f"decoded to max_length {args.e2e_len}",
                   "calls": args.e2e_calls, "prefill_s_per_call": pre_s / args.e2e_calls,
                   "verify_rounds_s_per_call": ver_s / args.e2e_calls, "rounds_per_call": rounds_total / args.e2e_calls}
    result = {
        "metric": METRIC, "value": accepted_all / (ms_max * 1e-3), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic: random-init weights N(0,0.02), uniform-random prompt ids",
        "config": workload_config(rows, args.prefix, spec.n_layers, world),
        "engine": {"lm_head": args.lm_head, "dense": args.dense,
                   "dense_shapes": {f"{k[0]}x{k[1]}x{k[2]}/{['store', 'resid', 'swiglu'][k[3]]}": v
                                    for k, v in eng.tile_report.items()},
                   "l2": "inputs larger than L2: 3.1 GB weights + KV cache re-read every step",
                   "graphs": "each step replays a captured CUDA graph of the round"},
        "accepted_tokens": accepted_all, "average_accept_length": accepted_all / (K * rows * world),
        "rollouts_gathered": int(lengths_all.numel()),
        "gpu_launches": launches_per_step * K,
        "roofline": {"kernel": "fg_tree_attention (fg::tc::attn_tc_kernel, tcgen05)", "bound": "hbm",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback", "traffic": traffic,
                     "algorithmic_bytes_per_launch": attn_bytes_b2b, "avg_launch_ms": attn_b2b_ms,
                     "launches_timed": 2 * spec.n_layers,
                     "timing": "CUDA events around 56 back-to-back launches of the round's attention call "
                               "over the 28 layers' KV caches (no L2 reuse), after the timed steps",
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


# ------------------------------------------------------------- CPU oracle
def cpu_oracle_round_rate(warm_rounds: int, timed_rounds: int, rows: int = 64, prefix: int = 1024):
    """The oracle's restatement of the reference generate loop on the host
    cores, on config 2's own shape (fp32): `rows` rollouts (rows / 8 prompts x
    8 samples) of `prefix`-token uniform-random prompts, the same tree plan
    (cpeak 1024, at most 16 nodes), HF eager attention with the dense tree
    mask.  The prefill is not timed; `timed_rounds` verify rounds after
    `warm_rounds` are."""
    import torch

    from oracle import reference_path as rp
    from flashgrpo_b200.utils import synthetic

    torch.set_num_threads(os.cpu_count() or 1)
    model = synthetic.build_model(2, device="cpu", dtype=torch.float32, attn_implementation="eager",
                                  fast_host_init=True)
    st = synthetic.medusa_head_tensors(2, dtype=torch.float32)

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
              "fc_w": st[f"heads.{i}.fc.weight"], "fc_b": st[f"heads.{i}.fc.bias"]} for i in range(3)]
    prompts = max(1, rows // 8)
    ids, mask = synthetic.random_prompts(prompts, prefix, 151936, seed=100)
    cfg = rp.OracleConfig(tree_mode="concurrency_aware", cpeak_nodes=1024, max_tree_nodes_per_seq=16,
                          max_tree_depth=4, fixed_tree_topk_by_depth=(4, 3, 2), top_p=1.0)
    t0 = time.perf_counter()
    res = rp.generate(model, heads, ids, mask, cfg, rp.SeqRoundSampler(1234), repeats=8,
                      max_length=prefix + warm_rounds + timed_rounds + 2, prefill_fn=synthetic_prefill)
    wall = time.perf_counter() - t0
    times = res["round_times"][warm_rounds:warm_rounds + timed_rounds]
    sec = sum(t for t, _ in times)
    tok = sum(n for _, n in times)
    return {"value": tok / sec, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(times)} verify rounds (after {warm_rounds} untimed) of config 2's full shape: "
                      f"{rows} rollouts ({prompts} prompts x 8 samples) with {prefix}-token prefixes, 28 layers, "
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
        base = cpu_oracle_round_rate(W, K, rows=args.rows, prefix=args.prefix)
        line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": args.gpus,
                "steps": K, "warmup": W, "ms_per_step": 1e3 * base["seconds"] / K, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic: random-init weights N(0,0.02), uniform-random prompt ids",
                "config": workload_config(args.rows, args.prefix, 28, args.gpus),
                "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
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
            result["cpu_baseline"] = cpu_oracle_round_rate(1, 3, rows=args.rows, prefix=args.prefix)
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""Generate golden fixtures by running the reference implementation on CPU.

Run in a container that has the reference checked out (read-only) at
``$FG_REFERENCE_ROOT`` (the ihbkaiser/ss-GRPO source tree):

    FG_REFERENCE_ROOT=/path/to/ss-GRPO python tests/golden/make_golden.py

It imports the reference's ``flashgrpo_b200`` package, runs its hot-path
functions on seeded inputs and writes small fixtures next to this script.
The fixtures pin the CPU oracle (``oracle/``) to the reference; the GPU box
only reads the fixtures and never needs the reference.

Two substitutions make the reference deterministic and comparable:
* ``torch.topk`` inside ``medusa_tree`` is replaced by a stable top-k (value
  descending, index ascending) -- torch leaves the tie order unspecified.
* ``sample_from_logits`` is replaced by the fg-icdf-v1 sampler of the C
  oracle fed with Philox uniforms; which uniform a row receives is recorded
  so the oracle walk can be replayed with the same draws.
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
if not os.environ.get("FG_REFERENCE_ROOT"):
    sys.exit("set FG_REFERENCE_ROOT to the root of the ihbkaiser/ss-GRPO source tree")
REF = Path(os.environ["FG_REFERENCE_ROOT"])
sys.path.insert(0, str(REF))
sys.path.insert(0, str(REPO))

from oracle import native  # noqa: E402

from flashgrpo_b200.decoding import acceptance as ref_acc  # noqa: E402  (reference package)
from flashgrpo_b200.decoding import flash_medusa_decoder as ref_dec  # noqa: E402
from flashgrpo_b200.decoding import medusa_tree as ref_tree  # noqa: E402
from flashgrpo_b200.decoding.kv_extraction import extract_accepted_path_kv  # noqa: E402
from flashgrpo_b200.decoding.tree_attention import build_tree_attention_inputs  # noqa: E402
from flashgrpo_b200.models.medusa_heads import MedusaHeads  # noqa: E402

_spec = importlib.util.spec_from_file_location("fg_synth", REPO / "ss-grpo_b200/flashgrpo_b200/utils/synthetic.py")
synth = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(synth)


class _StableTorch:
    """Proxy for the ``torch`` name inside medusa_tree with a stable topk."""

    def __getattr__(self, name):
        return getattr(torch, name)

    @staticmethod
    def topk(x, k, dim=-1, largest=True, sorted=True):
        assert largest and dim in (-1, x.dim() - 1)
        v, i = torch.sort(x, dim=-1, descending=True, stable=True)
        return torch.return_types.topk((v[..., :k], i[..., :k]))


ref_tree.torch = _StableTorch()
# the chain proposal's per-parent top-k (flash_medusa_decoder.py:1203) takes
# the same stable rule; the decoder's only other topk (:1028) reads values only
ref_dec.torch = _StableTorch()


def _bf16_logits(g, shape, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).float()


# ------------------------------------------------------------------ planner
def gen_planner():
    cases = []
    for mode in ("fixed", "concurrency_aware"):
        for bsz in (1, 16, 64, 256):
            for cpeak in (64, 1024, 4096):
                for mx in (10, 16, 32, 64):
                    for depth in (3, 5):
                        for topk in ((4, 3, 2), (4, 2, 2), (8, 8, 8, 8), (5, 4, 0)):
                            for adaptive, amin in ((False, (1, 1, 1)), (True, (1, 1, 1)), (True, (2, 2, 2, 2))):
                                if mode == "fixed" and adaptive:
                                    continue
                                kw = dict(active_batch_size=bsz, num_medusa_heads=4, tree_mode=mode,
                                          tree_layout="dense", cpeak_nodes=cpeak, min_tree_nodes_per_seq=1,
                                          max_tree_nodes_per_seq=mx, max_tree_depth=depth,
                                          fixed_tree_topk_by_depth=list(topk), adaptive_tree_enabled=adaptive,
                                          adaptive_min_topk_by_depth=list(amin))
                                p = ref_tree.plan_tree(**kw)
                                cases.append([mode, bsz, cpeak, mx, depth, list(topk), adaptive, list(amin),
                                              p.node_budget_per_seq, p.active_heads, list(p.topk_by_depth),
                                              p.actual_nodes])
    fits = []
    rng = np.random.default_rng(5)
    for _ in range(300):
        n = int(rng.integers(1, 6))
        topk = [int(x) for x in rng.integers(1, 9, n)]
        mins = [int(x) for x in rng.integers(1, 4, n)]
        budget = int(rng.integers(1, 80))
        decay = float(rng.choice([0.25, 0.5, 0.75, 1.0]))
        fits.append({"topk": topk, "budget": budget, "min": mins, "decay": decay,
                     "out": ref_tree.fit_topk_to_budget(topk, budget, min_topk_by_depth=mins,
                                                         depth_weight_decay=decay)})
    # adaptive mapping from confidences (decoder :1042-1061)
    conf_cases = []
    dec = ref_dec.FlashMedusaDecoder.__new__(ref_dec.FlashMedusaDecoder)
    for low, high in ((0.15, 0.45), (0.2, 0.2), (0.05, 0.9)):
        cfg = ref_dec.FlashMedusaConfig(adaptive_tree_enabled=True, adaptive_confidence_low=low,
                                        adaptive_confidence_high=high, adaptive_min_topk_by_depth=(1, 2, 1, 1))
        dec.config = cfg
        for c in np.linspace(0.0, 1.0, 41):
            for base in (1, 2, 4, 8):
                for d in range(4):
                    conf_cases.append({"low": low, "high": high, "min": [1, 2, 1, 1], "conf": float(c), "base": base,
                                       "depth": d, "out": dec._topk_from_confidence(float(c), base, d)})
    (HERE / "planner.json").write_text(json.dumps({"plans": cases, "fits": fits, "conf": conf_cases}))


# -------------------------------------------------------- trees and masks
def gen_trees():
    g = torch.Generator().manual_seed(11)
    out = {}
    plans = [
        ref_tree.TreePlan(16, 3, [4, 2, 2], 0, "fixed", "dense"),
        ref_tree.TreePlan(13, 2, [4, 2], 0, "concurrency_aware", "dense"),
        ref_tree.TreePlan(10, 3, [4, 3, 2], 0, "concurrency_aware", "dense"),
        ref_tree.TreePlan(32, 4, [3, 3, 2, 1], 0, "concurrency_aware", "dense"),
        ref_tree.TreePlan(64, 5, [2, 2, 2, 2, 2], 0, "concurrency_aware", "dense"),
        ref_tree.TreePlan(5, 1, [8], 0, "concurrency_aware", "dense"),
    ]
    for pi, plan in enumerate(plans):
        B, V = 6, 97
        root = torch.randint(0, V, (B,), generator=g)
        # coarse values force many ties, which the stable rule must resolve
        logits = [torch.round(torch.randn(B, V, generator=g) * 2) / 2 for _ in range(plan.active_heads)]
        trees = ref_tree.build_batch_trees(root, logits, plan)
        nmax = max(t.node_count for t in trees)
        full = torch.ones(B, 7, dtype=torch.long)
        full[1, :3] = 0
        logical = full.sum(-1)
        ids, mask4d, pos, node_mask = build_tree_attention_inputs(trees, full, logical, pad_token_id=0,
                                                                 dtype=torch.float32)
        out[f"p{pi}_root"] = root.numpy()
        out[f"p{pi}_logits"] = torch.stack(logits).numpy()
        out[f"p{pi}_plan"] = np.array([plan.node_budget_per_seq] + plan.topk_by_depth, dtype=np.int32)
        out[f"p{pi}_tokens"] = np.array([t.tokens + [-1] * (nmax - t.node_count) for t in trees], dtype=np.int32)
        out[f"p{pi}_parents"] = np.array([t.parents + [-2] * (nmax - t.node_count) for t in trees], dtype=np.int32)
        out[f"p{pi}_depths"] = np.array([t.depths + [1] * (nmax - t.node_count) for t in trees], dtype=np.int32)
        out[f"p{pi}_ids"] = ids.numpy()
        out[f"p{pi}_allowed"] = (mask4d == 0).numpy()
        out[f"p{pi}_pos"] = pos.numpy()
        out[f"p{pi}_node_mask"] = node_mask.numpy()
        out[f"p{pi}_full_mask"] = full.numpy()
        rows, nodes, slots = ref_dec.FlashMedusaDecoder._internal_tree_logit_layout(trees, device=torch.device("cpu"))
        out[f"p{pi}_slots"] = np.array(slots, dtype=np.int32)
    np.savez_compressed(HERE / "trees.npz", **out)


# ------------------------------------------------------------- acceptance
class _RecordingSampler:
    """fg-icdf-v1 sampler whose uniform is looked up from the logits row."""

    def __init__(self, table, uniforms):
        self.table = table  # bytes of a logits row -> (row, step)
        self.uniforms = uniforms

    def __call__(self, logits, *, do_sample=True, temperature=1.0, top_p=1.0, top_k=None, nucleus_topk_hint=2048):
        assert top_k is None and (top_p is None or top_p >= 1.0)
        x = logits.detach().float().numpy()
        u = np.array([self.uniforms[self.table[r.tobytes()]] for r in x], dtype=np.float32)
        return torch.from_numpy(native.sample_rows(x, u, do_sample=do_sample, temperature=temperature).astype(np.int64))


def gen_accept():
    g = torch.Generator().manual_seed(23)
    out = {}
    case = 0
    for V, B, temp, peaked, do_sample in ((64, 16, 1.0, 4.0, True), (97, 24, 0.7, 3.0, True), (4096, 8, 1.0, 8.0, True),
                                           (50, 12, 1.0, 1.0, False), (33, 20, 1.3, 6.0, True)):
        plan = ref_tree.TreePlan(16, 3, [4, 2, 2], 0, "fixed", "dense")
        root = torch.randint(0, V, (B,), generator=g)
        head_logits = [_bf16_logits(g, (B, V), peaked) for _ in range(3)]
        trees = ref_tree.build_batch_trees(root, head_logits, plan)
        rows, nodes, slots = ref_dec.FlashMedusaDecoder._internal_tree_logit_layout(trees, device=torch.device("cpu"))
        rows, nodes = rows.tolist(), nodes.tolist()
        # target logits correlated with the head logits so some paths get accepted
        packed = torch.stack([head_logits[min(int(trees[r].depths[n]) - 1, 2)][r] for r, n in zip(rows, nodes)])
        packed = (packed + _bf16_logits(g, packed.shape, 0.5)).to(torch.bfloat16).float()
        nmax = max(t.node_count for t in trees)
        uniforms = {}
        table = {}
        for r, n in zip(rows, nodes):
            step = int(trees[r].depths[n]) - 1
            table[packed[slots[r][n]].numpy().tobytes()] = (r, step)
        U = np.zeros((B, 4), dtype=np.float32)
        for r in range(B):
            for s in range(4):
                U[r, s] = native.uniform(99, r, case, 1 + s)
                uniforms[(r, s)] = U[r, s]
        ref_acc_orig = ref_acc.sample_from_logits
        ref_acc.sample_from_logits = _RecordingSampler(table, uniforms)
        try:
            acc, accn, par, corr = ref_acc.exact_accept_paths_batch(
                trees, packed, do_sample=do_sample, temperature=temp, top_p=1.0, top_k=None, node_to_logit_cpu=slots)
        finally:
            ref_acc.sample_from_logits = ref_acc_orig
        pre = f"c{case}_"
        out[pre + "meta"] = np.array([V, B, nmax, int(do_sample)], dtype=np.int32)
        out[pre + "temp"] = np.array([temp], dtype=np.float32)
        out[pre + "logits"] = packed.numpy()
        out[pre + "slots"] = np.array(slots, dtype=np.int32)
        out[pre + "tokens"] = np.array([t.tokens + [-1] * (nmax - t.node_count) for t in trees], dtype=np.int32)
        out[pre + "parents"] = np.array([t.parents + [-2] * (nmax - t.node_count) for t in trees], dtype=np.int32)
        out[pre + "n_nodes"] = np.array([t.node_count for t in trees], dtype=np.int32)
        out[pre + "uniforms"] = U
        dcap = 5
        out[pre + "acc_tokens"] = np.array([a + [-1] * (dcap - len(a)) for a in acc], dtype=np.int32)
        out[pre + "acc_nodes"] = np.array([a + [-1] * (dcap - len(a)) for a in accn], dtype=np.int32)
        out[pre + "parent"] = np.array(par, dtype=np.int32)
        out[pre + "correction"] = np.array([-1 if c is None else c for c in corr], dtype=np.int32)
        case += 1
    np.savez_compressed(HERE / "accept.npz", **out)


# -------------------------------------------------------------- extraction
def gen_extract():
    g = torch.Generator().manual_seed(31)
    out = {}
    for ci, (B, H, old, n, D, dtype) in enumerate(((3, 2, 9, 13, 8, torch.float32), (4, 2, 5, 16, 16, torch.bfloat16),
                                                  (2, 4, 1, 7, 64, torch.float32))):
        layers = []
        for _ in range(2):
            k = torch.randn(B, H, old + n, D, generator=g).to(dtype)
            v = torch.randn(B, H, old + n, D, generator=g).to(dtype)
            layers.append((k, v))
        paths = []
        for b in range(B):
            length = int(torch.randint(1, 5, (1,), generator=g))
            nodes = sorted(set([0] + torch.randint(1, n, (length - 1,), generator=g).tolist()))
            paths.append(nodes)
        old_cache = tuple((k[:, :, :old].clone(), v[:, :, :old].clone()) for k, v in layers)
        res = extract_accepted_path_kv(old_cache, tuple((k.clone(), v.clone()) for k, v in layers), paths,
                                       compact_in_place=True)
        pre = f"e{ci}_"
        out[pre + "meta"] = np.array([B, H, old, n, D, 1 if dtype == torch.bfloat16 else 0], dtype=np.int32)
        for li, (k, v) in enumerate(layers):
            out[pre + f"k{li}"] = k.view(torch.int16).numpy() if dtype == torch.bfloat16 else k.numpy()
            out[pre + f"v{li}"] = v.view(torch.int16).numpy() if dtype == torch.bfloat16 else v.numpy()
            rk, rv = res.past_key_values[li]
            out[pre + f"rk{li}"] = rk.contiguous().view(torch.int16).numpy() if dtype == torch.bfloat16 else rk.contiguous().numpy()
            out[pre + f"rv{li}"] = rv.contiguous().view(torch.int16).numpy() if dtype == torch.bfloat16 else rv.contiguous().numpy()
        out[pre + "paths"] = np.array([p + [-1] * (5 - len(p)) for p in paths], dtype=np.int32)
        out[pre + "max_len"] = np.array([res.max_accepted_length], dtype=np.int32)
    np.savez_compressed(HERE / "extract.npz", **out)


# ------------------------------------------------------- generate (config 1)
class _Tok:
    pad_token_id = 0
    eos_token_id = 1


class _CallOrderRefSampler:
    def __init__(self, seed):
        self.seed = seed
        self.calls = 0

    def __call__(self, logits, *, do_sample=True, temperature=1.0, top_p=1.0, top_k=None, nucleus_topk_hint=2048):
        x = logits.detach().float().numpy()
        u = np.array([native.uniform(self.seed, k, self.calls, 0) for k in range(x.shape[0])], dtype=np.float32)
        self.calls += 1
        # top_p < 1 / top_k: the fg-icdf-v1n / v1k draw from the kept set
        p = 1.0 if top_p is None else float(top_p)
        return torch.from_numpy(native.sample_rows(x, u, do_sample=do_sample, temperature=temperature,
                                                   top_p=p, top_k=top_k).astype(np.int64))


def gen_generate():
    results = {}
    runs = {
        "fixed_422": dict(tree_mode="fixed", fixed_tree_topk_by_depth=(4, 2, 2), max_tree_nodes_per_seq=16,
                          max_tree_depth=4, repeats=1, max_new=24, seed=0),
        "conc_rep2": dict(tree_mode="concurrency_aware", cpeak_nodes=64, fixed_tree_topk_by_depth=(4, 3, 2),
                          max_tree_nodes_per_seq=16, max_tree_depth=4, repeats=2, max_new=16, seed=3),
        "adaptive": dict(tree_mode="concurrency_aware", cpeak_nodes=128, fixed_tree_topk_by_depth=(8, 8, 8),
                         max_tree_nodes_per_seq=32, max_tree_depth=4, repeats=1, max_new=16, seed=5,
                         adaptive_tree_enabled=True, adaptive_min_topk_by_depth=(2, 2, 2)),
        # nucleus draws at the reference's default top_p
        "nucleus_095": dict(tree_mode="fixed", fixed_tree_topk_by_depth=(4, 2, 2), max_tree_nodes_per_seq=16,
                            max_tree_depth=4, repeats=1, max_new=20, seed=5, top_p=0.95),
        # chain proposals (_build_chain_batch_trees, :1141-1261) through the
        # ChainDraftCell, with the first state from MEDUSA head 1 and from the cell
        "chain_boot": dict(tree_mode="fixed", fixed_tree_topk_by_depth=(3, 2, 2), max_tree_nodes_per_seq=16,
                           max_tree_depth=4, repeats=1, max_new=20, seed=13, proposal_mode="chain",
                           chain_bootstrap_from_medusa=True),
        "chain_noboot": dict(tree_mode="fixed", fixed_tree_topk_by_depth=(2, 2), max_tree_nodes_per_seq=7,
                             max_tree_depth=3, repeats=2, max_new=16, seed=17, proposal_mode="chain",
                             chain_bootstrap_from_medusa=False),
        "chain_conc_p09": dict(tree_mode="concurrency_aware", cpeak_nodes=64, fixed_tree_topk_by_depth=(4, 3, 2),
                               max_tree_nodes_per_seq=16, max_tree_depth=4, repeats=2, max_new=16, seed=19,
                               proposal_mode="chain", chain_bootstrap_from_medusa=True, top_p=0.9),
        # top-k draws (sample_from_logits' top_k branch), alone and with top_p
        "topk_8": dict(tree_mode="fixed", fixed_tree_topk_by_depth=(4, 2, 2), max_tree_nodes_per_seq=16,
                       max_tree_depth=4, repeats=1, max_new=20, seed=23, top_k=8),
        "topk_40_p09": dict(tree_mode="concurrency_aware", cpeak_nodes=64, fixed_tree_topk_by_depth=(4, 3, 2),
                            max_tree_nodes_per_seq=16, max_tree_depth=4, repeats=2, max_new=16, seed=29, top_k=40,
                            top_p=0.9),
        # top-k draws with chain proposals
        "chain_topk16": dict(tree_mode="fixed", fixed_tree_topk_by_depth=(3, 2, 2), max_tree_nodes_per_seq=16,
                             max_tree_depth=4, repeats=1, max_new=16, seed=31, proposal_mode="chain",
                             chain_bootstrap_from_medusa=True, top_k=16),
    }
    model = synth.build_model(1)
    ids, mask = synth.random_prompts(4, 128, 4096, seed=0)
    for name, r in runs.items():
        chain = r.get("proposal_mode", "medusa") == "chain"
        head_state = synth.medusa_head_tensors(1, chain=chain)
        heads = MedusaHeads(256, 4096, 3, tie_lm_head=True)
        missing = heads.load_state_dict(head_state, strict=False)
        assert not missing.unexpected_keys
        cfg = ref_dec.FlashMedusaConfig(
            num_medusa_heads=3, tree_mode=r["tree_mode"], cpeak_nodes=r.get("cpeak_nodes", 512),
            max_tree_nodes_per_seq=r["max_tree_nodes_per_seq"], max_tree_depth=r["max_tree_depth"],
            fixed_tree_topk_by_depth=r["fixed_tree_topk_by_depth"], temperature=1.0, top_p=r.get("top_p", 1.0),
            top_k=r.get("top_k"),
            adaptive_tree_enabled=r.get("adaptive_tree_enabled", False),
            adaptive_min_topk_by_depth=r.get("adaptive_min_topk_by_depth", (1, 1, 1)),
            proposal_mode=r.get("proposal_mode", "medusa"),
            chain_bootstrap_from_medusa=r.get("chain_bootstrap_from_medusa", True),
            allow_recompute_fallback=False,
        )
        sampler = _CallOrderRefSampler(r["seed"])
        orig = (ref_dec.sample_from_logits, ref_acc.sample_from_logits)
        ref_dec.sample_from_logits = sampler
        ref_acc.sample_from_logits = sampler
        try:
            p_ids, p_mask = (ids[:2], mask[:2]) if r["repeats"] > 1 else (ids, mask)
            dec = ref_dec.FlashMedusaDecoder(model, heads, _Tok(), cfg)
            res = dec.generate(p_ids, p_mask, repeated_generate_nums=r["repeats"], max_length=128 + r["max_new"])
        finally:
            ref_dec.sample_from_logits, ref_acc.sample_from_logits = orig
        keep = ("generated_token_ids", "total_acc_length", "average_accept_length", "total_decoded_token_num",
                "total_verify_rounds", "total_correction_tokens", "total_accepted_medusa_tokens",
                "total_proposed_medusa_tokens", "kv_extraction_success_count", "kv_extraction_fallback_count")
        # every deterministic statistic (counts, histograms, plans; not the
        # timings) and the full key set, which the drop-in's result must cover
        stats = {k: v for k, v in res.items() if k not in keep and "time" not in k and not k.startswith("sampled_")
                 and k not in ("reflex_metrics", "reflex_head_metrics", "reflex_aux_records", "motivation_trace",
                               "persistent_memory_feedback", "last_tree_plan")}
        results[name] = {"run": {k: (list(v) if isinstance(v, tuple) else v) for k, v in r.items()},
                         **{k: res[k] for k in keep}, "stats": stats, "result_keys": sorted(res)}
    (HERE / "generate_cfg1.json").write_text(json.dumps(results))


# ------------------------------------------------------------------ nucleus
def gen_nucleus():
    """Kept sets of the reference's nucleus rule (logits_to_probs,
    acceptance.py:7-31: sort descending, keep through the first cumulative
    probability above top_p) on seeded rows with distinct logits, plus each
    row's distance between top_p and the reference's fp32 cumulative sums on
    either side of the boundary (rows where that distance is at the level of
    fp32 rounding may legitimately differ in the last kept entry)."""
    g = torch.Generator().manual_seed(2024)
    rows, temps, tops, kept, margin = [], [], [], [], []
    for r in range(48):
        V = [97, 512, 1000, 4096][r % 4]
        scale = [0.5, 1.0, 3.0, 8.0][(r // 4) % 4]
        logits = torch.randn(V, generator=g) * scale
        T = [1.0, 0.7, 1.3][r % 3]
        top_p = [0.5, 0.8, 0.9, 0.95, 0.99][r % 5]
        probs = ref_acc.logits_to_probs(logits[None], temperature=T, top_p=top_p)[0]
        sp = torch.softmax(logits.float() / T, dim=-1).sort(descending=True).values
        cum = torch.cumsum(sp, dim=-1)
        k = int((cum > top_p).nonzero()[0]) if bool((cum > top_p).any()) else V - 1
        lo = float(cum[k - 1]) if k > 0 else 0.0
        rows.append(np.pad(logits.numpy().astype(np.float32), (0, 4096 - V), constant_values=np.nan))
        temps.append(T)
        tops.append(top_p)
        kept.append(np.pad((probs > 0).numpy(), (0, 4096 - V)))
        margin.append(min(abs(float(cum[k]) - top_p), abs(lo - top_p)))
    np.savez_compressed(HERE / "nucleus.npz", logits=np.stack(rows), vocab=np.array([[97, 512, 1000, 4096][r % 4]
                        for r in range(48)], dtype=np.int32), temperature=np.array(temps, dtype=np.float32),
                        top_p=np.array(tops, dtype=np.float32), kept=np.stack(kept), margin=np.array(margin))


# -------------------------------------------------------------------- top-k
def gen_topk():
    """Kept sets of the reference's top-k rule on seeded rows with distinct
    logits: the tokens sample_from_logits' top_k branch (acceptance.py:68-79)
    hands to torch.multinomial with non-zero weight, captured at that call,
    and the non-zero entries of logits_to_probs (acceptance.py:7-31) with the
    same arguments, which must agree.  With 0 < top_p < 1 the row's margin is
    as in gen_nucleus, on the cumulative sums over the k candidates."""
    g = torch.Generator().manual_seed(2025)
    rows, temps, tops, ks, kept, margin = [], [], [], [], [], []
    seen = []
    real_multinomial = torch.multinomial

    def capture(weights, num_samples, *a, **kw):
        seen.append(weights.detach().clone())
        return real_multinomial(weights, num_samples, *a, **kw)

    for r in range(48):
        V = [97, 512, 1000, 4096][r % 4]
        scale = [0.5, 1.0, 3.0, 8.0][(r // 4) % 4]
        logits = torch.randn(V, generator=g) * scale
        T = [1.0, 0.7, 1.3][r % 3]
        top_k = [1, 2, 7, 40, 96][r % 5]
        top_p = [1.0, 0.9, 0.5, 0.95][(r // 2) % 4]
        seen.clear()
        torch.multinomial = capture
        try:
            ref_acc.sample_from_logits(logits[None], do_sample=True, temperature=T, top_p=top_p, top_k=top_k)
        finally:
            torch.multinomial = real_multinomial
        cand = torch.topk(logits[None], k=top_k, dim=-1, largest=True, sorted=True).indices[0]
        mask = np.zeros(V, dtype=bool)
        mask[cand[seen[0][0] > 0].numpy()] = True
        probs = ref_acc.logits_to_probs(logits[None], temperature=T, top_p=top_p, top_k=top_k)[0]
        assert np.array_equal(mask, (probs > 0).numpy()), r
        sp = torch.softmax(logits.float().topk(top_k).values / T, dim=-1)
        cum = torch.cumsum(sp, dim=-1)
        if 0.0 < top_p < 1.0:
            k = int((cum > top_p).nonzero()[0]) if bool((cum > top_p).any()) else top_k - 1
            lo = float(cum[k - 1]) if k > 0 else 0.0
            margin.append(min(abs(float(cum[k]) - top_p), abs(lo - top_p)))
        else:
            margin.append(1.0)
        rows.append(np.pad(logits.numpy().astype(np.float32), (0, 4096 - V), constant_values=np.nan))
        temps.append(T)
        tops.append(top_p)
        ks.append(top_k)
        kept.append(np.pad(mask, (0, 4096 - V)))
    np.savez_compressed(HERE / "topk.npz", logits=np.stack(rows), vocab=np.array([[97, 512, 1000, 4096][r % 4]
                        for r in range(48)], dtype=np.int32), temperature=np.array(temps, dtype=np.float32),
                        top_p=np.array(tops, dtype=np.float32), top_k=np.array(ks, dtype=np.int32),
                        kept=np.stack(kept), margin=np.array(margin))


GENERATORS = {"planner": lambda: gen_planner(), "trees": lambda: gen_trees(), "accept": lambda: gen_accept(),
              "extract": lambda: gen_extract(), "generate": lambda: gen_generate(), "nucleus": lambda: gen_nucleus(),
              "topk": lambda: gen_topk()}

if __name__ == "__main__":
    # python tests/golden/make_golden.py [name ...]  (default: every fixture)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    native.build()
    for name in (sys.argv[1:] or list(GENERATORS)):
        GENERATORS[name]()
    print("golden fixtures written to", HERE)

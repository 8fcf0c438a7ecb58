"""Random-init policies and prompts for the benchmark configurations.

No checkpoints or datasets exist offline, so tests and ``bench.py`` build
models of the named shapes with N(0, 0.02) weights from a fixed seed, and
prompts of uniform-random token ids.  This module imports only torch and
transformers so that fixture generators can load it by file path.

Shapes (configs of the benchmark):
  1  tiny Qwen2: 2 layers, hidden 256, 4/2 heads, head_dim 64, inter 688,
     vocab 4096, rope 1e6, fp32, lm_head scaled by 8, 3 MEDUSA heads.
  2  Qwen2.5-1.5B: 28 layers, hidden 1536, 12/2 heads, head_dim 128,
     inter 8960, vocab 151936, tied embeddings, bf16, 3 heads.
  3  Qwen2.5-7B: 28 layers, hidden 3584, 28/4, inter 18944, vocab 152064,
     4 heads.
  4  Llama-3.1-8B: 32 layers, hidden 4096, 32/8, inter 14336, vocab 128256,
     rope 5e5.
"""
from __future__ import annotations

import torch

CONFIGS = {
    1: dict(arch="qwen2", layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, inter=688, vocab=4096,
            rope_theta=1e6, dtype=torch.float32, lm_scale=8.0, medusa_heads=3, tie=False),
    2: dict(arch="qwen2", layers=28, hidden=1536, heads=12, kv_heads=2, head_dim=128, inter=8960, vocab=151936,
            rope_theta=1e6, dtype=torch.bfloat16, lm_scale=1.0, medusa_heads=3, tie=True),
    3: dict(arch="qwen2", layers=28, hidden=3584, heads=28, kv_heads=4, head_dim=128, inter=18944, vocab=152064,
            rope_theta=1e6, dtype=torch.bfloat16, lm_scale=1.0, medusa_heads=4, tie=False),
    4: dict(arch="llama", layers=32, hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=14336, vocab=128256,
            rope_theta=5e5, dtype=torch.bfloat16, lm_scale=1.0, medusa_heads=3, tie=False),
}


def hf_config(cfg_id: int, *, attn_implementation: str = "eager", **overrides):
    spec = dict(CONFIGS[cfg_id])
    spec.update(overrides)
    if spec["arch"] == "qwen2":
        from transformers import Qwen2Config as C
    else:
        from transformers import LlamaConfig as C
    conf = C(
        vocab_size=spec["vocab"],
        hidden_size=spec["hidden"],
        intermediate_size=spec["inter"],
        num_hidden_layers=spec["layers"],
        num_attention_heads=spec["heads"],
        num_key_value_heads=spec["kv_heads"],
        head_dim=spec["head_dim"],
        max_position_embeddings=65536,
        rope_theta=spec["rope_theta"],
        rms_norm_eps=1e-6,
        tie_word_embeddings=spec["tie"],
        initializer_range=0.02,
        attn_implementation=attn_implementation,
    )
    if spec["arch"] == "llama":
        conf.rope_parameters = {"rope_type": "default", "rope_theta": spec["rope_theta"]}
    return conf, spec


def _parallel_init(model, seed: int, std: float = 0.02):
    """HF's Qwen2 / Llama initialisation (Linear and Embedding weights
    N(0, std), biases 0, norm weights 1) filled by host threads: every
    parameter is cut into chunks, each drawn from its own seeded generator."""
    from concurrent.futures import ThreadPoolExecutor
    import os

    chunk = 1 << 24
    jobs = []
    for pi, (name, p) in enumerate(model.named_parameters()):
        flat = p.data.view(-1)
        if name.endswith("bias"):
            flat.zero_()
        elif "norm" in name:
            flat.fill_(1.0)
        else:
            for ci, off in enumerate(range(0, flat.numel(), chunk)):
                jobs.append((flat[off:off + chunk], seed * 1000003 + pi * 4099 + ci))

    def fill(job):
        t, sd = job
        g = torch.Generator().manual_seed(sd)
        t.normal_(0.0, std, generator=g)

    with ThreadPoolExecutor(max_workers=os.cpu_count() or 1) as ex:
        list(ex.map(fill, jobs))


def build_model(cfg_id: int, *, device="cpu", seed: int = 0, attn_implementation: str = "eager",
                fast_host_init: bool = False, **overrides):
    """Random-init causal LM of config ``cfg_id`` (weights N(0, 0.02), seeded).

    fast_host_init: build on the host with the weights drawn by parallel
    seeded generators (the same distribution, another random stream) instead
    of HF's single-threaded initialisation -- minutes faster for the 1.5B+
    shapes; used where only the shape matters (host timing baselines)."""
    conf, spec = hf_config(cfg_id, attn_implementation=attn_implementation, **overrides)
    if spec["arch"] == "qwen2":
        from transformers import Qwen2ForCausalLM as M
    else:
        from transformers import LlamaForCausalLM as M
    torch.manual_seed(seed)
    if fast_host_init:
        with torch.device("meta"):
            model = M(conf)
        model = model.to_empty(device="cpu").to(dtype=spec["dtype"])
        _parallel_init(model, seed)
        if hasattr(model, "tie_weights"):
            model.tie_weights()
        # the rotary embedding's non-persistent buffers are rebuilt from the config
        model.model.rotary_emb = type(model.model.rotary_emb)(config=model.config)
        model = model.eval()
    else:
        with torch.device(device):
            model = M(conf)
        model = model.to(dtype=spec["dtype"]).eval()
    if spec["lm_scale"] != 1.0:
        with torch.no_grad():
            model.lm_head.weight.mul_(spec["lm_scale"])
    return model


def medusa_head_tensors(cfg_id: int, *, device="cpu", seed: int = 1, dtype=None, chain: bool = False,
                        **overrides):
    """Parameters of the MEDUSA heads as plain tensors, keyed like the
    ``heads.{i}.norm`` / ``heads.{i}.fc`` entries of ``medusa_heads.pt``.

    fc weights are N(0, 0.02) (not the zero init of a fresh head) so the heads
    differ from the identity; LayerNorm weight 1 and bias 0.  chain=True adds
    the ``chain_cell.*`` entries of a ChainDraftCell (bottleneck max(64, H/8))
    with N(0, 0.02) projections, a non-zero out_proj and gate 0, so the cell
    changes the state.
    """
    spec = dict(CONFIGS[cfg_id])
    spec.update(overrides)
    H = spec["hidden"]
    dtype = dtype or spec["dtype"]
    g = torch.Generator(device="cpu").manual_seed(seed)
    state = {}
    for i in range(spec["medusa_heads"]):
        state[f"heads.{i}.fc.weight"] = (torch.randn(H, H, generator=g) * 0.02).to(device=device, dtype=dtype)
        state[f"heads.{i}.fc.bias"] = torch.zeros(H, device=device, dtype=dtype)
        state[f"heads.{i}.norm.weight"] = torch.ones(H, device=device, dtype=dtype)
        state[f"heads.{i}.norm.bias"] = torch.zeros(H, device=device, dtype=dtype)
    if chain:
        bn = max(64, H // 8)
        r = lambda *shape: (torch.randn(*shape, generator=g) * 0.02).to(device=device, dtype=dtype)
        state["chain_cell.state_norm.weight"] = torch.ones(H, device=device, dtype=dtype)
        state["chain_cell.state_norm.bias"] = torch.zeros(H, device=device, dtype=dtype)
        state["chain_cell.token_norm.weight"] = torch.ones(H, device=device, dtype=dtype)
        state["chain_cell.token_norm.bias"] = torch.zeros(H, device=device, dtype=dtype)
        state["chain_cell.state_proj.weight"] = r(bn, H)
        state["chain_cell.token_proj.weight"] = r(bn, H)
        state["chain_cell.out_proj.weight"] = r(H, bn) * 10
        state["chain_cell.out_proj.bias"] = torch.zeros(H, device=device, dtype=dtype)
        state["chain_cell.gate"] = torch.zeros((), device=device, dtype=dtype)
    return state


def random_prompts(n_prompts: int, length: int, vocab: int, *, seed: int = 0, low: int = 2):
    g = torch.Generator(device="cpu").manual_seed(seed)
    ids = torch.randint(low, vocab, (n_prompts, length), generator=g, dtype=torch.long)
    return ids, torch.ones_like(ids)

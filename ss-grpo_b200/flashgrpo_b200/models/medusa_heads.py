"""MEDUSA heads: nn.Module mirror of flashgrpo_b200/models/medusa_heads.py.

Parameter names and shapes match the reference so ``medusa_heads.pt``
checkpoints load unchanged (``heads.{i}.fc``, ``heads.{i}.norm``,
``chain_cell.*``; :699-774 for the save/load format).  The modules keep a
plain PyTorch forward for callers that use them directly; the B200 verify
engine reads their weights and runs the heads with its own kernels
(``fg_layernorm`` / ``fg_silu_residual`` around a cuBLAS GEMM).
"""
from __future__ import annotations

import json
from pathlib import Path

import torch
import torch.nn as nn
import torch.nn.functional as F


class ChainDraftCell(nn.Module):
    """state + sigmoid(gate) * W_out SiLU(W_s LN(state) + W_t LN(embedding)) (medusa_heads.py:130-160)."""

    def __init__(self, hidden_size: int, *, bottleneck_ratio: int = 8, gate_init: float = -3.0, dtype=None):
        super().__init__()
        hidden_size = int(hidden_size)
        bottleneck = max(64, hidden_size // max(1, int(bottleneck_ratio)))
        self.state_norm = nn.LayerNorm(hidden_size, dtype=dtype)
        self.token_norm = nn.LayerNorm(hidden_size, dtype=dtype)
        self.state_proj = nn.Linear(hidden_size, bottleneck, bias=False, dtype=dtype)
        self.token_proj = nn.Linear(hidden_size, bottleneck, bias=False, dtype=dtype)
        self.out_proj = nn.Linear(bottleneck, hidden_size, bias=True, dtype=dtype)
        self.gate = nn.Parameter(torch.tensor(float(gate_init), dtype=dtype or torch.float32))
        nn.init.zeros_(self.out_proj.weight)
        nn.init.zeros_(self.out_proj.bias)

    def forward(self, state: torch.Tensor, token_embedding: torch.Tensor) -> torch.Tensor:
        dt = self.state_norm.weight.dtype
        s = state.to(dt)
        mixed = self.state_proj(self.state_norm(s)) + self.token_proj(self.token_norm(token_embedding.to(dt)))
        return s + torch.sigmoid(self.gate) * self.out_proj(F.silu(mixed))


class MedusaPredictionHead(nn.Module):
    """h + SiLU(fc(LayerNorm(h))) followed by the (tied) lm_head (medusa_heads.py:211-256)."""

    def __init__(self, hidden_size: int, vocab_size: int, *, dtype=None, tie_lm_head: bool = True, lm_head=None):
        super().__init__()
        self.hidden_size = int(hidden_size)
        self.vocab_size = int(vocab_size)
        self.tie_lm_head = bool(tie_lm_head)
        self.fc = nn.Linear(hidden_size, hidden_size, bias=True, dtype=dtype)
        self.norm = nn.LayerNorm(hidden_size, dtype=dtype)
        nn.init.zeros_(self.fc.weight)
        nn.init.zeros_(self.fc.bias)
        self.output = None
        if not self.tie_lm_head:
            self.output = nn.Linear(hidden_size, vocab_size, bias=False, dtype=dtype)
            if lm_head is not None and getattr(lm_head, "weight", None) is not None \
                    and lm_head.weight.shape == self.output.weight.shape:
                with torch.no_grad():
                    self.output.weight.copy_(lm_head.weight.detach().to(self.output.weight.dtype))

    def project_hidden(self, hidden_states: torch.Tensor) -> torch.Tensor:
        x = hidden_states.to(self.norm.weight.dtype)
        return x + F.silu(self.fc(self.norm(x)))

    def forward(self, hidden_states: torch.Tensor, lm_head=None) -> torch.Tensor:
        h = self.project_hidden(hidden_states)
        if self.output is not None:
            return self.output(h)
        if lm_head is None:
            raise ValueError("lm_head is required when tie_lm_head=True")
        bias = getattr(lm_head, "bias", None)
        return F.linear(h.to(lm_head.weight.dtype), lm_head.weight.detach(), None if bias is None else bias.detach())


class MedusaHeads(nn.Module):
    def __init__(self, hidden_size: int, vocab_size: int, num_heads: int = 3, *, dtype=None, tie_lm_head: bool = True,
                 lm_head=None, medusa_loss_decay: float = 0.8, chain_bottleneck_ratio: int = 8,
                 chain_gate_init: float = -3.0, **unused_reflex_kwargs):
        super().__init__()
        self.hidden_size = int(hidden_size)
        self.vocab_size = int(vocab_size)
        self.num_heads = int(num_heads)
        self.tie_lm_head = bool(tie_lm_head)
        self.medusa_loss_decay = float(medusa_loss_decay)
        self.chain_bottleneck_ratio = int(chain_bottleneck_ratio)
        self.chain_gate_init = float(chain_gate_init)
        self.heads = nn.ModuleList([
            MedusaPredictionHead(hidden_size, vocab_size, dtype=dtype, tie_lm_head=tie_lm_head, lm_head=lm_head)
            for _ in range(self.num_heads)
        ])
        self.chain_cell = ChainDraftCell(hidden_size, bottleneck_ratio=chain_bottleneck_ratio,
                                         gate_init=chain_gate_init, dtype=dtype)

    def project_hidden_for_head(self, hidden_states: torch.Tensor, head_idx: int, **_unused) -> torch.Tensor:
        return self.heads[max(0, min(int(head_idx), len(self.heads) - 1))].project_hidden(hidden_states)

    def forward(self, hidden_states: torch.Tensor, lm_head=None, *, max_heads: int | None = None):
        heads = self.heads if max_heads is None else self.heads[: max(0, min(int(max_heads), len(self.heads)))]
        return [head(hidden_states, lm_head=lm_head) for head in heads]

    def logits_for_last_hidden(self, last_hidden: torch.Tensor, lm_head=None, *, max_heads: int | None = None,
                               **_unused) -> list[torch.Tensor]:
        if last_hidden.dim() == 2:
            last_hidden = last_hidden.unsqueeze(1)
        n = len(self.heads) if max_heads is None else max(0, min(int(max_heads), len(self.heads)))
        return [self.heads[i](last_hidden, lm_head=lm_head)[:, -1, :] for i in range(n)]

    def chain_next_state(self, state: torch.Tensor, token_ids: torch.Tensor, embedding_layer) -> torch.Tensor:
        return self.chain_cell(state, embedding_layer(token_ids.to(state.device)).detach())

    def chain_logits_from_state(self, state: torch.Tensor, lm_head) -> torch.Tensor:
        bias = getattr(lm_head, "bias", None)
        return F.linear(state.to(lm_head.weight.dtype), lm_head.weight.detach(), None if bias is None else bias.detach())

    def save_pretrained(self, save_directory) -> None:
        d = Path(save_directory)
        d.mkdir(parents=True, exist_ok=True)
        config = {"hidden_size": self.hidden_size, "vocab_size": self.vocab_size, "num_heads": self.num_heads,
                  "tie_lm_head": self.tie_lm_head, "medusa_loss_decay": self.medusa_loss_decay,
                  "chain_bottleneck_ratio": self.chain_bottleneck_ratio, "chain_gate_init": self.chain_gate_init}
        (d / "medusa_config.json").write_text(json.dumps(config, indent=2), encoding="utf-8")
        try:
            import yaml

            (d / "medusa_config.yaml").write_text(yaml.safe_dump(config, sort_keys=False), encoding="utf-8")
        except ImportError:  # pragma: no cover - yaml is optional
            pass
        torch.save(self.state_dict(), d / "medusa_heads.pt")

    @classmethod
    def from_pretrained(cls, load_directory, *, map_location="cpu", dtype=None, lm_head=None,
                        chain_bottleneck_ratio=None, chain_gate_init=None, **_unused) -> "MedusaHeads":
        d = Path(load_directory)
        config = json.loads((d / "medusa_config.json").read_text(encoding="utf-8"))
        model = cls(config["hidden_size"], config["vocab_size"], config["num_heads"], dtype=dtype,
                    tie_lm_head=config.get("tie_lm_head", True), lm_head=lm_head,
                    medusa_loss_decay=config.get("medusa_loss_decay", 0.8),
                    chain_bottleneck_ratio=(chain_bottleneck_ratio if chain_bottleneck_ratio is not None
                                            else config.get("chain_bottleneck_ratio", 8)),
                    chain_gate_init=(chain_gate_init if chain_gate_init is not None
                                     else config.get("chain_gate_init", -3.0)))
        state = torch.load(d / "medusa_heads.pt", map_location=map_location)
        current = model.state_dict()
        compatible = {k: v for k, v in state.items() if k in current and tuple(current[k].shape) == tuple(v.shape)}
        model.load_state_dict(compatible, strict=False)
        model._loaded_state_keys = set(state.keys())
        model._loaded_compatible_keys = set(compatible.keys())
        return model

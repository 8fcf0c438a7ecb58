"""HF plugin for the tree attention kernel: ``attn_implementation="fg_tree"``.

The reference's tree forward (``models/qwen_flashgrpo_wrapper.py:220-239``)
runs an HF decoder with eager/SDPA attention over a ``DynamicCache`` and a
dense additive 4D mask built by ``build_tree_attention_inputs``
(``decoding/tree_attention.py:6-67``).  Importing this module registers
``"fg_tree"`` in HF's ``AttentionInterface``; a model whose
``config._attn_implementation`` is ``"fg_tree"``, called with

    model(input_ids=tree_tokens, position_ids=tree_positions,
          past_key_values=cache,                  # FGStaticCache
          fg_tree=TreeInputs(cache, anc_bits))    # forwarded to every attention call

then runs ``fg_tree_attention`` in every layer: the cache writes each layer's
tree K/V at each row's own length (no padding holes, nothing appended), and
the kernel reads the row's prefix plus the tree through the ancestor bits --
no dense mask is built (HF skips mask creation for attention functions without
a mask function).  The cache's lengths are not advanced: acceptance decides
which tree slots survive (``fg_extract_path`` / ``fg_accept_extract``).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from transformers import AttentionInterface
from transformers.cache_utils import Cache

from .. import ops


class FGStaticCache(Cache):
    """Preallocated K/V ``[layers][B][Hkv][capacity][D]`` with per-row lengths
    ``row_len`` (int32 on the device): row b's prefix is slots
    ``[0, row_len[b])``; ``update`` writes a forward's new tokens at slots
    ``row_len[b] + j``."""

    def __init__(self, k: torch.Tensor, v: torch.Tensor, row_len: torch.Tensor):
        super().__init__(layers=[])
        if k.shape != v.shape or k.dim() != 5:
            raise ValueError("k and v must be [layers, B, Hkv, capacity, D] tensors of one shape")
        if row_len.dtype != torch.int32 or row_len.shape != (k.shape[1],):
            raise ValueError("row_len must be int32 [B]")
        self.k, self.v, self.row_len = k, v, row_len
        self.kv_layers = [ops.kv_layer(k[l], v[l]) for l in range(k.shape[0])]

    @classmethod
    def empty(cls, n_layers: int, batch: int, n_kv_heads: int, capacity: int, head_dim: int, *, dtype, device):
        k = torch.zeros((n_layers, batch, n_kv_heads, capacity, head_dim), dtype=dtype, device=device)
        return cls(k, torch.zeros_like(k), torch.zeros(batch, dtype=torch.int32, device=device))

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        """key/value ``[B, Hkv, n, D]`` (RoPE applied) -> slots
        ``row_len[b] + j`` of layer ``layer_idx``; returns that layer's cache."""
        B, _, n, _ = key_states.shape
        # clamped so the write stays inside the cache; the attention of layer
        # 0 rejects a forward that does not fit (row_len + n <= capacity)
        pos = (self.row_len.long()[:, None] + torch.arange(n, device=key_states.device)[None, :]).clamp_(
            max=self.k.shape[3] - 1)
        rows = torch.arange(B, device=key_states.device)[:, None].expand(B, n)
        self.k[layer_idx][rows, :, pos] = key_states.permute(0, 2, 1, 3).to(self.k.dtype)
        self.v[layer_idx][rows, :, pos] = value_states.permute(0, 2, 1, 3).to(self.v.dtype)
        return self.k[layer_idx], self.v[layer_idx]

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return int(self.row_len.max()) if self.row_len.numel() else 0

    def get_max_cache_shape(self, layer_idx: int = 0) -> int:
        return self.k.shape[3]

    def __len__(self) -> int:
        return self.k.shape[0]


def ancestor_bits(parents: list[int], device=None) -> torch.Tensor:
    """int32 ``[N, 4]`` bits of node i's ancestors and itself (the attention
    rule of ``build_tree_attention_inputs``), for ``N <= 128`` nodes in
    topological order (parent index < child index)."""
    n = len(parents)
    if n > 128:
        raise ValueError("at most 128 tree nodes")
    words = [[0, 0, 0, 0] for _ in range(n)]
    for i, p in enumerate(parents):
        if p >= 0:
            words[i] = list(words[p])
        words[i][i >> 5] |= 1 << (i & 31)
    t = torch.tensor([[w - (1 << 32) if w >= 1 << 31 else w for w in row] for row in words], dtype=torch.int32)
    return t.to(device) if device is not None else t


@dataclass
class TreeInputs:
    """What the fg_tree attention needs besides Q: the cache (K/V and the
    per-row prefix lengths), the shared tree topology as ancestor bits and
    an optional split-K workspace (fg_tree_attention_workspace_size bytes,
    zero-filled; allocated on first use when omitted)."""

    cache: FGStaticCache
    anc_bits: torch.Tensor
    workspace: torch.Tensor | None = None
    num_splits: int = 0


def fg_tree_attention_forward(module, query, key, value, attention_mask, scaling=None, dropout=0.0, fg_tree=None,
                              **kwargs):
    """HF attention-function signature: query ``[B, Hq, N, D]`` -> output
    ``[B, N, Hq, D]``, no attention weights."""
    if fg_tree is None:
        raise ValueError("attn_implementation='fg_tree' needs fg_tree=TreeInputs(...) in the model call")
    if dropout:
        raise ValueError("fg_tree attention has no dropout")
    cache, layer = fg_tree.cache, module.layer_idx
    q = query.transpose(1, 2).contiguous()
    B, n, hq, D = q.shape
    hkv = cache.k.shape[2]
    if layer == 0 and int(cache.row_len.max()) + n > cache.k.shape[3]:
        raise ValueError("FGStaticCache capacity exceeded: row_len + tree nodes > capacity")
    if fg_tree.workspace is None:
        need = ops.attention_workspace_bytes(B, n, hq, hkv, D, num_splits=fg_tree.num_splits,
                                             max_kv_len=cache.k.shape[3])
        fg_tree.workspace = torch.zeros(max(need, 16) // 4 + 4, dtype=torch.int32, device=q.device)
    scale = scaling if scaling is not None else D ** -0.5
    out = ops.tree_attention(q, cache.k[layer], cache.v[layer], cache.row_len, fg_tree.anc_bits, scale=scale,
                             workspace=fg_tree.workspace, num_splits=fg_tree.num_splits,
                             max_kv_len=cache.k.shape[3], kv=cache.kv_layers[layer])
    return out, None


AttentionInterface.register("fg_tree", fg_tree_attention_forward)

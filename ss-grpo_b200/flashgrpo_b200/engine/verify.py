"""Verify engine: one MEDUSA tree-verify round on a B200, device resident.

A round (flashgrpo_b200/decoding/flash_medusa_decoder.py:1649-2938 of the
reference, Reflex off) runs as one stream of work with no host sync:

  propose   fg_medusa_propose: X = [h ; head_1(h) ; ... ; head_k(h)], the
            tied lm_head over X with the head rows' top-k fused       (K1)
            root token  = fg_sample_rows(root logits, forced = pending correction)
            chain proposals: one fg_chain_step per tree level (cell + top-k)
  tree      fg_build_tree: plan, dense tree, ancestor bits, slots     (K2)
  verify    per layer: RMSNorm, QKV GEMM (+bias), fg_rope_kv_write (RoPE +
            tree K/V written at each row's cache tail), fg_tree_attention
            (K3), O GEMM + residual, RMSNorm, gate/up GEMM with SwiGLU in
            the epilogue, down GEMM + residual (bf16: every GEMM is
            fg_linear, tcgen05 with the bias / residual / SwiGLU fused);
            final RMSNorm
  lm_head   internal (has-children) nodes only                  (fg_linear)
  accept    fg_accept_extract: exact_target walk, clip/EOS/pending rules,
            KV compaction in every layer, next hidden state           (K4)

State lives on the device between rounds: the KV cache
[layers, B, Hkv, capacity, D] with one logical length per row (no holes --
the reference's padded slots and attention-mask holes disappear), the next
round's hidden state (rows [0, B) of X), pending correction tokens, the
round counter feeding the Philox uniforms, and the active-row flags.

Because every tensor of a round has a fixed shape for a given (rows, plan),
the round is captured once in a CUDA graph and replayed.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _native as N
from .. import ops
from ..decoding.medusa_tree import TreePlan, dense_topology, internal_nodes, max_adaptive_internal


# ------------------------------------------------------------------ weights
@dataclass
class ModelSpec:
    n_layers: int
    hidden: int
    n_q_heads: int
    n_kv_heads: int
    head_dim: int
    inter: int
    vocab: int
    eps: float
    dtype: torch.dtype


def unwrap_causal_lm(causal_lm):
    if hasattr(causal_lm, "get_base_model"):
        return causal_lm.get_base_model()
    if hasattr(causal_lm, "base_model") and hasattr(causal_lm.base_model, "model"):
        return causal_lm.base_model.model
    return causal_lm


def _fuse_rows(modules_params: list[torch.nn.Parameter]) -> torch.Tensor:
    """Concatenates parameters along dim 0 and rebinds each one as a view of
    the fused tensor, so the HF model keeps working without a second copy."""
    fused = torch.cat([p.data for p in modules_params], 0).contiguous()
    off = 0
    for p in modules_params:
        n = p.shape[0]
        p.data = fused[off:off + n]
        off += n
    return fused


class TargetWeights:
    """The HF causal LM's parameters in the layout the verify forward uses."""

    def __init__(self, causal_lm):
        base = unwrap_causal_lm(causal_lm)
        core = base.model
        cfg = base.config
        hq = cfg.num_attention_heads
        self.spec = ModelSpec(
            n_layers=cfg.num_hidden_layers, hidden=cfg.hidden_size, n_q_heads=hq,
            n_kv_heads=cfg.num_key_value_heads, head_dim=getattr(cfg, "head_dim", None) or cfg.hidden_size // hq,
            inter=cfg.intermediate_size, vocab=cfg.vocab_size, eps=float(cfg.rms_norm_eps),
            dtype=next(base.parameters()).dtype)
        self.embed = core.embed_tokens.weight
        self.final_norm = core.norm.weight
        self.lm_head = base.lm_head.weight
        rot = core.rotary_emb
        self.inv_freq = rot.inv_freq.float().contiguous()
        self.attention_scaling = float(getattr(rot, "attention_scaling", 1.0))
        self.layers = []
        for layer in core.layers:
            at, mlp = layer.self_attn, layer.mlp
            qkv_b = None
            if at.q_proj.bias is not None:
                qkv_b = _fuse_rows([at.q_proj.bias, at.k_proj.bias, at.v_proj.bias])
            self.layers.append({
                "in_norm": layer.input_layernorm.weight,
                "w_qkv": _fuse_rows([at.q_proj.weight, at.k_proj.weight, at.v_proj.weight]),
                "b_qkv": qkv_b,
                "w_o": at.o_proj.weight,
                "b_o": at.o_proj.bias,
                "post_norm": layer.post_attention_layernorm.weight,
                "w_gu": _fuse_rows([mlp.gate_proj.weight, mlp.up_proj.weight]),
                "w_down": mlp.down_proj.weight,
            })


class HeadWeights:
    """MEDUSA head parameters (heads.{i}.norm / heads.{i}.fc of medusa_heads.pt)
    cast once to the model's compute dtype."""

    def __init__(self, heads, dtype, device):
        state = heads.state_dict() if hasattr(heads, "state_dict") else dict(heads)
        self.heads = []
        i = 0
        while f"heads.{i}.fc.weight" in state:
            g = lambda k: state[f"heads.{i}.{k}"].detach().to(device=device, dtype=dtype).contiguous()
            self.heads.append({"norm_w": g("norm.weight"), "norm_b": g("norm.bias"), "fc_w": g("fc.weight"),
                               "fc_b": g("fc.bias")})
            i += 1
        # ChainDraftCell (chain_cell.*), present when the checkpoint has one
        cell = {k[len("chain_cell."):]: v.detach().to(device=device, dtype=dtype) for k, v in state.items()
                if k.startswith("chain_cell.")}
        self.chain = cell if "state_proj.weight" in cell else None
        if any(k.startswith("heads.") and k.endswith("output.weight") for k in state):
            raise NotImplementedError("untied MEDUSA output heads are not on the B200 path (tie_lm_head=True)")

    def __len__(self):
        return len(self.heads)


# -------------------------------------------------------------- round state
@dataclass
class RoundConfig:
    do_sample: bool = True
    temperature: float = 1.0
    top_p: float = 1.0  # 0 < top_p < 1: nucleus draws (fg-icdf-v1n)
    top_k: int = 0  # 0 < top_k < vocab: top-k draws (fg-icdf-v1k); otherwise no cut
    eos_id: int = 1
    max_length: int = 1 << 30
    seed: int = 0
    attn_splits: int = 0
    # chain proposals (ChainDraftCell): per-parent top-k instead of per-head
    chain: bool = False
    chain_bootstrap: bool = True
    # proposal lm_head: "fused" = tcgen05 GEMM with the top-k in its epilogue
    # (bf16, hidden a multiple of 64, <= 256 rows), "separate" = cuBLAS GEMM
    # then fg_row_topk
    lm_head: str = "separate"
    # acceptance: every internal node's draw before the walk (one CTA per
    # packed logits row) instead of one draw per walk step; faster once the
    # walk visits more nodes than one wave of those CTAs covers
    parallel_draws: bool = False
    # verify-forward projections and the internal-node lm_head: "native" =
    # fg_linear (tcgen05, fused bias / residual / SwiGLU epilogues, bf16),
    # "cublas" = torch addmm / mm (+ fg_silu_mul), "auto" = per projection
    # shape whichever of the two measured faster on this GPU (fp32 always
    # uses cuBLAS)
    dense: str = "auto"


class DecodeState:
    """Device state of a batch of rollouts between rounds."""

    def __init__(self, spec: ModelSpec, B: int, capacity: int, device, n_heads: int):
        self.B, self.capacity = B, capacity
        L, hkv, D = spec.n_layers, spec.n_kv_heads, spec.head_dim
        # zero-filled once: every slot the attention kernel can touch is finite
        self.k = torch.zeros((L, B, hkv, capacity, D), dtype=spec.dtype, device=device)
        self.v = torch.zeros_like(self.k)
        self.row_len = torch.zeros(B, dtype=torch.int32, device=device)
        self.pending = torch.full((B,), -1, dtype=torch.int32, device=device)
        self.active = torch.ones(B, dtype=torch.int32, device=device)
        self.seq_ids = torch.arange(B, dtype=torch.int32, device=device)
        self.round_dev = torch.zeros(1, dtype=torch.int32, device=device)
        self.X = torch.zeros(((n_heads + 1) * B, spec.hidden), dtype=spec.dtype, device=device)
        self.kv_layers = [ops.kv_layer(self.k[l], self.v[l]) for l in range(L)]

    @property
    def hidden(self) -> torch.Tensor:
        return self.X[: self.B]


class RoundView:
    """The active rows of a DecodeState as a compact batch for one round:
    finished rows are retired without moving any K/V (the replacement of
    select_cache_batch, qwen_flashgrpo_wrapper.py:100-118).  Round row i is
    state row rows[i]; the per-row scalars and the hidden state are gathered
    before the round and scattered back after it (a few hundred KB), while
    the RoPE/KV write, the tree attention and the extract_path compaction
    address the shared cache through the row map.  It has DecodeState's
    attributes, so a round runs on it unchanged."""

    def __init__(self, st: DecodeState, B: int, n_heads: int):
        dev = st.row_len.device
        self.base = st
        self.B, self.capacity = B, st.capacity
        self.rows = torch.zeros(B, dtype=torch.int32, device=dev)
        self.row_len = torch.zeros(B, dtype=torch.int32, device=dev)
        self.pending = torch.full((B,), -1, dtype=torch.int32, device=dev)
        self.active = torch.ones(B, dtype=torch.int32, device=dev)
        self.seq_ids = torch.zeros(B, dtype=torch.int32, device=dev)
        self.round_dev = st.round_dev  # the round counter is shared by all rows
        self.X = torch.zeros(((n_heads + 1) * B, st.X.shape[1]), dtype=st.X.dtype, device=dev)
        self.k, self.v = st.k, st.v
        self.kv_layers = [ops.kv_layer(st.k[l], st.v[l], rows=self.rows) for l in range(st.k.shape[0])]

    @property
    def hidden(self) -> torch.Tensor:
        return self.X[: self.B]

    def gather(self):
        st, idx = self.base, self.rows.long()
        torch.index_select(st.row_len, 0, idx, out=self.row_len)
        torch.index_select(st.pending, 0, idx, out=self.pending)
        torch.index_select(st.active, 0, idx, out=self.active)
        torch.index_select(st.seq_ids, 0, idx, out=self.seq_ids)
        torch.index_select(st.hidden, 0, idx, out=self.hidden)

    def scatter(self):
        st, idx = self.base, self.rows.long()
        st.row_len.index_copy_(0, idx, self.row_len)
        st.pending.index_copy_(0, idx, self.pending)
        st.active.index_copy_(0, idx, self.active)
        st.hidden.index_copy_(0, idx, self.hidden)


class RoundBuffers:
    """Every intermediate of one round for a fixed (rows, plan) shape."""

    def __init__(self, spec: ModelSpec, B: int, plan: TreePlan, n_heads: int, device, dcap: int,
                 adaptive: bool = False):
        H, V = spec.hidden, spec.vocab
        self.n_heads = n_heads
        parents, depths = dense_topology(plan, n_heads)
        # BFS levels of the shared topology: level d = nodes at depth d + 1
        self.widths = [int(k) for k in plan.topk_by_depth[:n_heads]]
        self.level_off, self.level_count = [], []
        for d in range(1, max(depths, default=1) + 1):
            ids = [i for i, dd in enumerate(depths) if dd == d]
            self.level_off.append(ids[0] if ids else len(depths))
            self.level_count.append(len(ids))
        self.chain_tokens = []
        self.N = len(parents)
        self.internal = internal_nodes(parents)
        self.n_int = len(self.internal)
        self.kmax = max([int(k) for k in plan.topk_by_depth[:n_heads]] + [1])
        self.n_draws = 1 + max(len(plan.topk_by_depth), 1)
        N_, f = self.N, dict(device=device)
        self.logits = torch.empty(((n_heads + 1) * B, V), dtype=spec.dtype, **f)
        self.ln = torch.empty((B, H), dtype=spec.dtype, **f)
        self.fc = torch.empty((B, H), dtype=spec.dtype, **f)
        self.U = torch.empty((B, self.n_draws), dtype=torch.float32, **f)
        self.root = torch.empty(B, dtype=torch.int32, **f)
        hb = max(n_heads, 1) * B
        # the logsumexp is only consumed by adaptive trees
        self.topk = (torch.empty((hb, self.kmax), dtype=torch.int32, **f),
                     torch.empty((hb, self.kmax), dtype=torch.float32, **f),
                     torch.empty(hb, dtype=torch.float32, **f),
                     torch.empty(hb, dtype=torch.float32, **f) if adaptive else None)
        i32 = dict(dtype=torch.int32, **f)
        self.tree = {"tokens": torch.empty((B, N_), **i32), "positions": torch.empty((B, N_), **i32),
                     "slot": torch.empty((B, N_), **i32), "parents": torch.empty(N_, **i32),
                     "depths": torch.empty(N_, **i32), "anc": torch.empty((N_, 4), **i32),
                     "internal": torch.empty(N_, **i32), "plan": torch.empty(16, **i32)}
        T = B * N_
        qkv_dim = (spec.n_q_heads + 2 * spec.n_kv_heads) * spec.head_dim
        self.h = torch.empty((T, H), dtype=spec.dtype, **f)
        self.xn = torch.empty((T, H), dtype=spec.dtype, **f)
        self.qkv = torch.empty((T, qkv_dim), dtype=spec.dtype, **f)
        self.q = torch.empty((B, N_, spec.n_q_heads, spec.head_dim), dtype=spec.dtype, **f)
        self.attn = torch.empty_like(self.q)
        self.gu = torch.empty((T, 2 * spec.inter), dtype=spec.dtype, **f)
        self.act = torch.empty((T, spec.inter), dtype=spec.dtype, **f)
        self.tree_hidden = torch.empty((B, N_, H), dtype=spec.dtype, **f)
        self.rope_cs = torch.empty((2, B * N_, spec.head_dim // 2), dtype=spec.dtype, **f)
        idx = [b * N_ + i for b in range(B) for i in self.internal]
        self.int_idx = torch.tensor(idx if idx else [0], dtype=torch.int32, **f)
        # Adaptive rounds keep this (base plan) shape: the tree that K2 builds
        # is never larger, its unused nodes are inert (parent -2, no slot),
        # and the internal-row gather is rebuilt on the device from K2's
        # internal list each round.
        # internal rows an adaptive tree can have: a narrower, deeper tree may
        # have more internal nodes than the base plan's own
        self.adaptive = adaptive
        n_rows = B * max_adaptive_internal(plan, n_heads) if adaptive else len(idx)
        self.j_int = torch.arange(max(n_rows, 1), dtype=torch.int32, **f)
        if adaptive:
            self.int_idx = torch.zeros(max(n_rows, 1), dtype=torch.int32, **f)
        self.hid_int = torch.empty((max(n_rows, 1), H), dtype=spec.dtype, **f)
        self.tree_logits = torch.empty((max(n_rows, 1), V), dtype=spec.dtype, **f)
        self.dcap = dcap
        # the acceptance walk's draws, one per packed internal-node logits row
        self.drawn = torch.empty(max(n_rows, 1), **i32)
        self.out = {k: torch.empty((B, dcap), **i32) for k in ("acc_tokens", "acc_nodes")}
        for k in ("acc_len", "correction", "last_node", "finished"):
            self.out[k] = torch.empty(B, **i32)
        self.acc_sum = torch.zeros(1, dtype=torch.int64, **f)
        ws = ops.attention_workspace_bytes(B, N_, spec.n_q_heads, spec.n_kv_heads, spec.head_dim, num_splits=0,
                                           max_kv_len=0)
        self.ws_bytes = ws
        self.attn_ws = None


# ------------------------------------------------------------------- engine
class VerifyEngine:
    def __init__(self, causal_lm, medusa_heads, *, device=None, autotune: bool = True, dense: str = "auto"):
        self.model = causal_lm
        # time fg_linear's tilings once per projection shape (else the library's choice)
        self.autotune = autotune
        # "auto": per shape, fg_linear or cuBLAS, whichever the tuning measured faster
        self.dense_mode = dense
        self.tile_report: dict = {}
        self.w = TargetWeights(causal_lm)
        self.spec = self.w.spec
        self.device = device or self.w.embed.device
        if self.device.type != "cuda":
            raise RuntimeError("VerifyEngine runs on a CUDA device (B200); the model is on " + str(self.device))
        N.load()
        self.heads = HeadWeights(medusa_heads, self.spec.dtype, self.device)
        self.scale = self.spec.head_dim ** -0.5
        self._graphs: dict = {}

    # -------------------------------------------------------------- prefill
    def state(self, B: int, capacity: int, n_heads: int) -> DecodeState:
        """A decode state of this shape, reused across calls (so captured
        round graphs stay valid) and reset for a new batch."""
        key = ("state", B, capacity, n_heads)
        st = self._graphs.get(key)
        if st is None:
            st = DecodeState(self.spec, B, capacity, self.device, n_heads)
            self._graphs[key] = st
        st.row_len.zero_()
        st.pending.fill_(-1)
        st.active.fill_(1)
        st.seq_ids.copy_(torch.arange(B, dtype=torch.int32, device=self.device))
        st.round_dev.zero_()
        return st

    @torch.no_grad()
    def prefill(self, input_ids, attention_mask, *, repeats: int = 1, capacity: int, n_heads: int) -> DecodeState:
        """Runs the HF model over the prompts, then moves the valid (non-pad)
        prompt K/V into the cache, repeated `repeats` times per prompt
        (flash_medusa_decoder.py:1325-1346)."""
        from transformers import DynamicCache

        base = unwrap_causal_lm(self.model)
        ids = input_ids.to(self.device, non_blocking=True)
        mask = attention_mask.to(self.device, non_blocking=True).long()
        pos = (mask.cumsum(-1) - 1).masked_fill(mask == 0, 0)
        out = base.model(input_ids=ids, attention_mask=mask, position_ids=pos, past_key_values=DynamicCache(),
                         use_cache=True, return_dict=True)
        hid = out.last_hidden_state
        n_valid = mask.sum(-1)
        P, S = ids.shape
        B = P * repeats
        if int(n_valid.max()) + 1 > capacity:  # the one host sync of the prefill
            raise ValueError("KV capacity smaller than the prompt")
        st = self.state(B, capacity, n_heads)
        # valid (mask == 1) positions first, in order: slot j of a row holds its
        # j-th valid token; slots past the row's length hold finite padding K/V
        order = torch.argsort((mask == 0).to(torch.int8), dim=-1, stable=True)
        W = min(S, capacity)
        for l, layer in enumerate(out.past_key_values.layers):
            for src, dst in ((layer.keys, st.k), (layer.values, st.v)):
                idx = order[:, None, :W, None].expand(-1, src.shape[1], -1, src.shape[3])
                dst[l, :, :, :W] = torch.gather(src, 2, idx).repeat_interleave(repeats, 0)
        last = (mask * torch.arange(S, device=mask.device)).argmax(-1)  # last valid position
        last = torch.where(n_valid > 0, last, torch.full_like(last, S - 1))
        st.X[:B] = hid[torch.arange(P, device=hid.device), last].repeat_interleave(repeats, 0)
        st.row_len[:B] = n_valid.to(torch.int32).repeat_interleave(repeats)
        del out
        return st

    # ---------------------------------------------------------------- round
    def buffers(self, B: int, plan: TreePlan, n_heads: int, dcap: int, adaptive: bool = False) -> RoundBuffers:
        key = ("buf", B, plan.node_budget_per_seq, tuple(plan.topk_by_depth), n_heads, dcap, adaptive)
        if key not in self._graphs:
            self._graphs[key] = RoundBuffers(self.spec, B, plan, n_heads, self.device, dcap, adaptive)
        return self._graphs[key]

    def _fused_lm_head(self, cfg: RoundConfig, M: int) -> bool:
        sp = self.spec
        return (cfg.lm_head == "fused" and sp.dtype == torch.bfloat16 and sp.hidden % 64 == 0 and M <= 256
                and self.w.lm_head.stride(1) == 1)

    def _lm_head_ws(self, M: int, topk_row0: int, k: int) -> torch.Tensor:
        need = ops.lm_head_topk_workspace_bytes(M, self.spec.vocab, topk_row0, k)
        ws = getattr(self, "_lmh_ws", None)
        if ws is None or ws.numel() * 4 < need:
            ws = torch.empty(max(need, 16) // 4 + 64, dtype=torch.int32, device=self.device)
            self._lmh_ws = ws
        return ws

    def _attn_workspace(self, rb: RoundBuffers, st: DecodeState, splits: int):
        need = ops.attention_workspace_bytes(st.B, rb.N, self.spec.n_q_heads, self.spec.n_kv_heads,
                                             self.spec.head_dim, num_splits=splits, max_kv_len=st.capacity)
        if need and (rb.attn_ws is None or rb.attn_ws.numel() * 4 < need):
            rb.attn_ws = torch.zeros(need // 4 + 64, dtype=torch.int32, device=self.device)
        return rb.attn_ws

    def _native_dense(self, cfg: RoundConfig) -> bool:
        """fg_linear can run this model's projections (bf16, K multiples of 64)
        and the round asks for it ("native", or "auto" per shape)."""
        sp = self.spec
        return (cfg.dense in ("native", "auto") and sp.dtype == torch.bfloat16 and sp.hidden % 64 == 0
                and sp.inter % 64 == 0 and (sp.n_q_heads * sp.head_dim) % 64 == 0 and self.w.lm_head.stride(1) == 1
                and self.w.lm_head.stride(0) == sp.hidden)

    # ---------------------------------------------------- dense projections
    @staticmethod
    def _tile_ok(pair: bool, bn: int, epi: int) -> bool:
        """fg_linear's tile rule: the epilogue's 32-column TMEM reads stay in
        the tile's 256-column accumulator; an SM pair splits the weight rows
        in two 8-row-aligned halves."""
        nb = 2 * bn if epi == ops.EPI_SWIGLU else bn
        if bn % 16 or nb > 256 or (pair and (nb // 2) % 8):
            return False
        return bn // 2 + (bn // 2 + 31) // 32 * 32 + (bn if epi == ops.EPI_SWIGLU else 0) <= 256

    def _tune_linear(self, M: int, n_out: int, K: int, epi: int):
        """The fastest fg_linear tiling (token rows, outputs, k ranges) of one
        projection shape, timed with CUDA events on random
        operands whose weights rotate through more copies than L2 holds (the
        round reads every layer's weights from HBM).  Runs once per shape,
        outside any stream capture."""
        dev = self.device
        rows = 2 * n_out if epi == ops.EPI_SWIGLU else n_out
        nk = K // 64
        cands = []
        for pair in (False, True):
            for bn in range(48, 257, 16):
                if not self._tile_ok(pair, bn, epi) or (epi == ops.EPI_SWIGLU and n_out % bn):
                    continue
                n_units = -(-M // (256 if pair else 128)) * -(-n_out // bn)
                for sp in (1, 2, 3, 4, 6, 8):
                    if sp > 1 and nk // sp < 4:
                        break
                    if n_units * sp > 24 * 148:
                        continue
                    nb = 2 * bn if epi == ops.EPI_SWIGLU else bn
                    stage = 128 * 128 + (nb // 2 if pair else nb) * 128
                    for st in ((6,) if pair else (4, 6, 8)):
                        if st * stage <= 227 * 1024 - 2048:
                            cands.append((256 if pair else 128, bn, sp, st))
        if not cands:
            return (0, 0, 0, 0)
        g = torch.Generator(device=dev).manual_seed(1)
        copies = max(1, min(16, -(-(256 << 20) // (rows * K * 2))))
        ws_ = [torch.randn(rows, K, generator=g, device=dev, dtype=torch.bfloat16) * 0.02 for _ in range(copies)]
        x = torch.randn(M, K, generator=g, device=dev, dtype=torch.bfloat16)
        b = torch.zeros(n_out, device=dev, dtype=torch.bfloat16) if epi == ops.EPI_STORE else None
        h = torch.zeros(M, n_out, device=dev, dtype=torch.bfloat16)
        need = max(ops.linear_workspace_bytes(M, n_out, K, epi, bn, sp, bm) for bm, bn, sp, _ in cands)
        wsp = torch.zeros(need // 4 + 64, dtype=torch.int32, device=dev) if need else None

        def timed(c, reps=8):
            # the launches are replayed from a CUDA graph, so the device time
            # is measured, not the host's launch rate
            bm, bn, sp, st = c
            run = lambda i: ops.linear(x, ws_[i % copies], bias=b, resid=h if epi == ops.EPI_RESID else None, out=h,
                                       epilogue=epi, bm=bm, bn=bn, splits=sp, stages=st, workspace=wsp)
            run(0)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(reps):
                    run(i + 1)
            graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize(dev)
            return e0.elapsed_time(e1) / reps

        res = sorted((timed(c), c) for c in cands)
        best = res[0][1]
        self.tile_report[(M, n_out, K, epi)] = {"fg_linear_us": 1e3 * res[0][0], "tile": list(best)}
        if self.dense_mode == "auto":
            # the library GEMM with the same epilogue, timed the same way
            gu = torch.empty(M, 2 * n_out, device=dev, dtype=torch.bfloat16) if epi == ops.EPI_SWIGLU else None

            def cublas(i):
                w_ = ws_[i % copies]
                if epi == ops.EPI_SWIGLU:
                    torch.mm(x, w_.t(), out=gu)
                    ops.silu_mul(gu, out=h)
                elif epi == ops.EPI_RESID:
                    torch.addmm(h, x, w_.t(), out=h)
                else:
                    torch.addmm(b, x, w_.t(), out=h) if b is not None else torch.mm(x, w_.t(), out=h)

            cublas(0)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(8):
                    cublas(i + 1)
            graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize(dev)
            t_cub = e0.elapsed_time(e1) / 8
            self.tile_report[(M, n_out, K, epi)]["cublas_us"] = 1e3 * t_cub
            if t_cub < res[0][0]:
                best = None
        self.tile_report[(M, n_out, K, epi)]["uses"] = "fg_linear" if best is not None else "cublas"
        del ws_, x, h, wsp
        return best

    def _tile(self, M: int, n_out: int, K: int, epi: int):
        """The fg_linear tiling of a projection shape, or None where the
        round runs that shape on cuBLAS ("auto" measured it faster).  Shapes
        are tuned per 128-row bucket of M (the tile grid is the same for
        every M of a bucket, for 128- and 256-row tiles alike), so a round
        whose active rows shrink by a few retired rows reuses the decision
        instead of timing the candidates again."""
        Mb = -(-M // 128) * 128
        key = ("tile", Mb, n_out, K, epi)
        if key not in self._graphs:
            self._graphs[key] = self._tune_linear(Mb, n_out, K, epi) if self.autotune else (0, 0, 0, 0)
        return self._graphs[key]

    def _linear(self, x, w, *, epi, bias=None, resid=None, out=None, gu=None):
        """One projection: fg_linear with this shape's tuned tiling and
        workspace, or the cuBLAS form of the same epilogue."""
        M, K = x.shape
        n_out = w.shape[0] // 2 if epi == ops.EPI_SWIGLU else w.shape[0]
        tile = self._tile(M, n_out, K, epi)
        if tile is None:
            if epi == ops.EPI_SWIGLU:
                torch.mm(x, w.t(), out=gu)
                return ops.silu_mul(gu, out=out)
            if epi == ops.EPI_RESID:
                torch.addmm(resid, x, w.t(), out=out)
                if bias is not None:
                    out.add_(bias)
                return out
            return torch.addmm(bias, x, w.t(), out=out) if bias is not None else torch.mm(x, w.t(), out=out)
        bm, bn, sp, st = tile
        return ops.linear(x, w, bias=bias, resid=resid, out=out, epilogue=epi, bm=bm, bn=bn, splits=sp, stages=st,
                          workspace=self._linear_ws(M, n_out, K, epi))

    def _linear_ws(self, M: int, n_out: int, K: int, epi: int):
        """Zero-filled split-K workspace of one projection shape (None when its
        tiling needs none); one per shape, reused by every layer in turn."""
        tile = self._tile(M, n_out, K, epi)
        if tile is None:
            return None
        bm, bn, sp, _ = tile
        need = ops.linear_workspace_bytes(M, n_out, K, epi, bn, sp, bm)
        if not need:
            return None
        key = ("linws", M, n_out, K, epi)
        ws = self._graphs.get(key)
        if ws is None or ws.numel() * 4 < need:
            ws = torch.zeros(need // 4 + 64, dtype=torch.int32, device=self.device)
            self._graphs[key] = ws
        return ws

    def _prepare_linear(self, rb: "RoundBuffers", B: int):
        """Allocates the round's projection workspaces (before any capture)."""
        sp = self.spec
        T = B * rb.N
        qkv = (sp.n_q_heads + 2 * sp.n_kv_heads) * sp.head_dim
        self._linear_ws(T, qkv, sp.hidden, ops.EPI_STORE)
        self._linear_ws(T, sp.hidden, sp.n_q_heads * sp.head_dim, ops.EPI_RESID)
        self._linear_ws(T, sp.inter, sp.hidden, ops.EPI_SWIGLU)
        self._linear_ws(T, sp.hidden, sp.inter, ops.EPI_RESID)
        self._linear_ws(rb.hid_int.shape[0], sp.vocab, sp.hidden, ops.EPI_STORE)

    def _propose_ws(self, B: int, nh: int, k: int) -> torch.Tensor:
        need = ops.medusa_propose_workspace_bytes(B, self.spec.hidden, self.spec.vocab, nh, k)
        ws = getattr(self, "_prop_ws", None)
        if ws is None or ws.numel() * 4 < need:
            ws = torch.empty(max(need, 16) // 4 + 64, dtype=torch.int32, device=self.device)
            self._prop_ws = ws
        return ws

    def propose(self, st: DecodeState, rb: RoundBuffers, cfg: RoundConfig):
        B, nh = st.B, rb.n_heads
        h = st.hidden
        M = (nh + 1) * B
        if self._fused_lm_head(cfg, M):
            # heads and lm_head in one call: root rows keep their logits (the
            # sampler reads them); head rows only produce their top-k
            ops.medusa_propose(st.X[:M], B, self.heads.heads[:nh], self.w.lm_head, root_logits=rb.logits,
                               k=rb.kmax, topk_out=rb.topk if nh > 0 else None,
                               workspace=self._propose_ws(B, nh, rb.kmax))
        else:
            for i in range(nh):
                hw = self.heads.heads[i]
                ops.layernorm(h, hw["norm_w"], hw["norm_b"], 1e-5, out=rb.ln)
                torch.addmm(hw["fc_b"], rb.ln, hw["fc_w"].t(), out=rb.fc)
                ops.silu_residual(h, rb.fc, out=st.X[(i + 1) * B:(i + 2) * B])
            torch.mm(st.X[:M], self.w.lm_head.t(), out=rb.logits[:M])
            if nh > 0:
                ops.row_topk(rb.logits[B:M], rb.kmax, out=rb.topk)
        ops.philox_uniforms(cfg.seed, st.seq_ids, 0, rb.n_draws, out=rb.U, round_dev=st.round_dev)
        ops.sample_rows(rb.logits[:B], rb.U, do_sample=cfg.do_sample, temperature=cfg.temperature,
                        top_p=cfg.top_p, top_k=cfg.top_k, forced=st.pending, out=rb.root)

    # ------------------------------------------------------ chain proposals
    def _chain_cell(self, state: torch.Tensor, emb: torch.Tensor) -> torch.Tensor:
        """ChainDraftCell.forward (medusa_heads.py:154-160) in the cell's dtype."""
        F = torch.nn.functional
        c = self.heads.chain
        H = state.shape[-1]
        mixed = (F.linear(F.layer_norm(state, (H,), c["state_norm.weight"], c["state_norm.bias"], 1e-5),
                          c["state_proj.weight"])
                 + F.linear(F.layer_norm(emb, (H,), c["token_norm.weight"], c["token_norm.bias"], 1e-5),
                            c["token_proj.weight"]))
        delta = F.linear(F.silu(mixed), c["out_proj.weight"], c["out_proj.bias"])
        return state + torch.sigmoid(c["gate"]) * delta

    def _rows_topk(self, x: torch.Tensor, k: int, cfg: RoundConfig) -> torch.Tensor:
        """Stable top-k indices [M, k] of the lm_head logits of the rows of x."""
        M, V = x.shape[0], self.spec.vocab
        idx = torch.empty((M, k), dtype=torch.int32, device=self.device)
        val = torch.empty((M, k), dtype=torch.float32, device=self.device)
        mx = torch.empty(M, dtype=torch.float32, device=self.device)
        if self._fused_lm_head(cfg, min(M, 256)):
            for r0 in range(0, M, 256):
                r1 = min(M, r0 + 256)
                ws = self._lm_head_ws(r1 - r0, 0, k)
                ops.lm_head_topk(x[r0:r1], self.w.lm_head, n_logit_rows=0, logits=None, topk_row0=0, k=k,
                                 topk_out=(idx[r0:r1], val[r0:r1], mx[r0:r1], None), workspace=ws)
        else:
            logits = torch.mm(x, self.w.lm_head.t())
            ops.row_topk(logits, k, out=(idx, val, mx, None))
        return idx

    def _fused_chain(self, cfg: RoundConfig) -> bool:
        c, sp = self.heads.chain, self.spec
        return (cfg.lm_head == "fused" and sp.dtype == torch.bfloat16 and sp.hidden % 64 == 0
                and sp.hidden <= 8192 and c["state_proj.weight"].shape[0] % 64 == 0
                and self.w.lm_head.stride(1) == 1 and self.w.embed.stride(1) == 1)

    def _chain_ws(self, M: int, k: int) -> torch.Tensor:
        sp = self.spec
        need = ops.chain_step_workspace_bytes(M, sp.hidden, self.heads.chain["state_proj.weight"].shape[0],
                                              sp.vocab, k)
        ws = getattr(self, "_chain_ws_buf", None)
        if ws is None or ws.numel() * 4 < need:
            ws = torch.empty(max(need, 16) // 4 + 64, dtype=torch.int32, device=self.device)
            self._chain_ws_buf = ws
        return ws

    def _chain_topk_bufs(self, M: int, k: int):
        return (torch.empty((M, k), dtype=torch.int32, device=self.device),
                torch.empty((M, k), dtype=torch.float32, device=self.device),
                torch.empty(M, dtype=torch.float32, device=self.device), None)

    def propose_chain(self, st: DecodeState, rb: RoundBuffers, cfg: RoundConfig):
        """_build_chain_batch_trees (flash_medusa_decoder.py:1141-1261), Reflex
        off, fixed widths: the root token as in propose(), then per depth the
        lm_head top-k of every parent state and the chain cell on the chosen
        tokens.  The dense topology is the one K2 builds; the tokens of each
        level are written over K2's after build_tree.  bf16: each level is one
        fg_chain_step (cell + lm_head top-k of the new states), and a
        head-bootstrapped state comes from fg_medusa_propose with the root
        logits."""
        B = st.B
        h = st.hidden
        H = h.shape[-1]
        fused = self._fused_chain(cfg) and len(rb.widths) > 0
        idx = None
        if fused and cfg.chain_bootstrap and len(self.heads) > 0 and 2 * B <= 256:
            # root logits, head-0 state and its top-k in one call
            if st.X.shape[0] >= 2 * B:
                x2 = st.X[:2 * B]
            else:
                x2 = torch.empty((2 * B, H), dtype=h.dtype, device=self.device)
                x2[:B].copy_(h)
            k0 = rb.widths[0]
            top = self._chain_topk_bufs(B, k0)
            ops.medusa_propose(x2, B, self.heads.heads[:1], self.w.lm_head, root_logits=rb.logits, k=k0,
                               topk_out=top, workspace=self._propose_ws(B, 1, k0))
            state, idx = x2[B:], top[0]
        elif self._fused_lm_head(cfg, B):
            ops.lm_head_topk(st.X[:B], self.w.lm_head, n_logit_rows=B, logits=rb.logits, topk_row0=B, k=1,
                             topk_out=None, workspace=self._lm_head_ws(B, B, 1))
        else:
            torch.mm(st.X[:B], self.w.lm_head.t(), out=rb.logits[:B])
        ops.philox_uniforms(cfg.seed, st.seq_ids, 0, rb.n_draws, out=rb.U, round_dev=st.round_dev)
        ops.sample_rows(rb.logits[:B], rb.U, do_sample=cfg.do_sample, temperature=cfg.temperature,
                        top_p=cfg.top_p, top_k=cfg.top_k, forced=st.pending, out=rb.root)
        if idx is None:  # the state was not bootstrapped together with the root logits
            if cfg.chain_bootstrap and len(self.heads) > 0:
                hw = self.heads.heads[0]
                ops.layernorm(h, hw["norm_w"], hw["norm_b"], 1e-5, out=rb.ln)
                torch.addmm(hw["fc_b"], rb.ln, hw["fc_w"].t(), out=rb.fc)
                state = ops.silu_residual(h, rb.fc)
            elif fused:
                # the cell on the root token, with the depth-0 top-k
                k0 = rb.widths[0]
                state = torch.empty((B, H), dtype=h.dtype, device=self.device)
                top = self._chain_topk_bufs(B, k0)
                ops.chain_step(h, rb.root.view(B, 1), n_parent=1, fanout=1, n_child=1, embed=self.w.embed,
                               cell=self.heads.chain, lm_head=self.w.lm_head, k=k0, state_out=state, topk_out=top,
                               workspace=self._chain_ws(B, k0))
                idx = top[0]
            else:
                state = self._chain_cell(h, self.w.embed[rb.root.long()])
        states, n_par = state.reshape(B, 1, H), 1
        rb.chain_tokens = []
        for d, k in enumerate(rb.widths):
            n_ch = rb.level_count[d + 1] if d + 1 < len(rb.level_count) else 0
            if n_ch == 0:
                break
            if idx is None:
                idx = self._rows_topk(states.reshape(B * n_par, H), k, cfg)
            tok = idx.view(B, n_par * k)[:, :n_ch]
            rb.chain_tokens.append((rb.level_off[d + 1], n_ch, tok))
            if d + 2 < len(rb.level_count) and rb.level_count[d + 2] > 0:
                if fused and d + 1 < len(rb.widths):
                    k1 = rb.widths[d + 1]
                    new = torch.empty((B * n_ch, H), dtype=h.dtype, device=self.device)
                    top = self._chain_topk_bufs(B * n_ch, k1)
                    ops.chain_step(states.reshape(B * n_par, H), idx.view(B, n_par * k), n_parent=n_par, fanout=k,
                                   n_child=n_ch, embed=self.w.embed, cell=self.heads.chain, lm_head=self.w.lm_head,
                                   k=k1, state_out=new, topk_out=top, workspace=self._chain_ws(B * n_ch, k1))
                    states, idx = new.view(B, n_ch, H), top[0]
                else:
                    par = torch.arange(n_ch, device=self.device) // k
                    emb = self.w.embed[tok.reshape(-1).long()]
                    states = self._chain_cell(states[:, par].reshape(-1, H), emb).view(B, n_ch, H)
                    idx = None
                n_par = n_ch
            else:
                idx = None

    def build_tree(self, st: DecodeState, rb: RoundBuffers, params: N.PlanParams):
        nh = rb.n_heads
        B = st.B
        if nh > 0:
            cidx = rb.topk[0].view(nh, B, rb.kmax)
            cval = rb.topk[1].view(nh, B, rb.kmax)
            hmax = rb.topk[2].view(nh, B)
            hlse = rb.topk[3].view(nh, B) if rb.topk[3] is not None else None
        else:
            cidx = cval = hmax = hlse = None
        ops.build_tree(params, rb.root, cidx, cval, hmax, hlse, nmax=rb.N, logits_dtype=self.spec.dtype,
                       row_len=st.row_len, out=rb.tree)

    def verify_forward(self, st: DecodeState, rb: RoundBuffers, cfg: RoundConfig, attn_events=None):
        """attn_events (optional): per-layer (start, end) CUDA events recorded
        around the tree-attention launch, for live per-launch timing (None
        entries skip a layer; an event between the RoPE/KV write and the
        attention keeps that layer's attention from starting early)."""
        sp, w = self.spec, self.w
        B, N_ = st.B, rb.N
        ops.gather_rows(w.embed, rb.tree["tokens"].view(-1), out=rb.h)
        # the tree positions are fixed for the round: one cos/sin table for all layers
        ops.rope_table(rb.tree["positions"], w.inv_freq, w.attention_scaling, sp.dtype, out=rb.rope_cs)
        ws = self._attn_workspace(rb, st, cfg.attn_splits)
        # bf16: every projection on fg_linear with its consumer in the
        # epilogue (bias, residual add, SwiGLU); fp32 keeps cuBLAS
        native = self._native_dense(cfg)
        T = B * N_
        if native:
            self._prepare_linear(rb, B)
        for l, lw in enumerate(w.layers):
            ops.rmsnorm(rb.h, lw["in_norm"], sp.eps, out=rb.xn)
            if native:
                self._linear(rb.xn, lw["w_qkv"], epi=ops.EPI_STORE, bias=lw["b_qkv"], out=rb.qkv)
            elif lw["b_qkv"] is not None:
                torch.addmm(lw["b_qkv"], rb.xn, lw["w_qkv"].t(), out=rb.qkv)
            else:
                torch.mm(rb.xn, lw["w_qkv"].t(), out=rb.qkv)
            kv = st.kv_layers[l]
            ops.rope_kv_write(rb.qkv, rb.tree["positions"], w.inv_freq, w.attention_scaling, B=B, n_nodes=N_,
                              n_q_heads=sp.n_q_heads, n_kv_heads=sp.n_kv_heads, head_dim=sp.head_dim,
                              kv_len=st.row_len, k_cache=None, v_cache=None, q_out=rb.q, kv=kv, cos_sin=rb.rope_cs)
            if attn_events is not None and attn_events[l] is not None:
                attn_events[l][0].record()
            ops.tree_attention(rb.q, st.k[l], st.v[l], st.row_len, rb.tree["anc"], scale=self.scale, out=rb.attn,
                               workspace=ws, num_splits=cfg.attn_splits, max_kv_len=st.capacity, kv=kv)
            if attn_events is not None and attn_events[l] is not None:
                attn_events[l][1].record()
            if native:
                self._linear(rb.attn.view(T, -1), lw["w_o"], epi=ops.EPI_RESID, bias=lw["b_o"], resid=rb.h, out=rb.h)
            else:
                torch.addmm(rb.h, rb.attn.view(T, -1), lw["w_o"].t(), out=rb.h)
                if lw["b_o"] is not None:
                    rb.h.add_(lw["b_o"])
            ops.rmsnorm(rb.h, lw["post_norm"], sp.eps, out=rb.xn)
            if native:
                self._linear(rb.xn, lw["w_gu"], epi=ops.EPI_SWIGLU, out=rb.act, gu=rb.gu)
                self._linear(rb.act, lw["w_down"], epi=ops.EPI_RESID, resid=rb.h, out=rb.h)
            else:
                torch.mm(rb.xn, lw["w_gu"].t(), out=rb.gu)
                ops.silu_mul(rb.gu, out=rb.act)
                torch.addmm(rb.h, rb.act, lw["w_down"].t(), out=rb.h)
        ops.rmsnorm(rb.h, w.final_norm, sp.eps, out=rb.tree_hidden.view(B * N_, -1))

    def accept(self, st: DecodeState, rb: RoundBuffers, cfg: RoundConfig, phase_event=None):
        """Internal-node logits, then K4.  phase_event (optional) is recorded
        between the two: the end of the verify phase."""
        B = st.B
        if rb.n_int > 0:
            if rb.adaptive:
                # row b * ni + rank -> tree_hidden[b, internal[rank]] (ni = this round's internal count)
                ni = rb.tree["plan"][11:12].clamp_min(1)
                b = torch.div(rb.j_int, ni, rounding_mode="floor")
                r = rb.j_int - b * ni
                idx = b * rb.N + rb.tree["internal"][r.long()]
                torch.where(rb.j_int < B * ni, idx, torch.zeros_like(idx), out=rb.int_idx)
            ops.gather_rows(rb.tree_hidden.view(B * rb.N, -1), rb.int_idx, out=rb.hid_int)
            if self._native_dense(cfg):
                self._linear(rb.hid_int, self.w.lm_head, epi=ops.EPI_STORE, out=rb.tree_logits)
            else:
                torch.mm(rb.hid_int, self.w.lm_head.t(), out=rb.tree_logits)
        if phase_event is not None:
            phase_event.record()
        outs = dict(rb.out)
        outs["pending"] = st.pending
        ops.accept_extract(logits=rb.tree_logits, slot=rb.tree["slot"], tokens=rb.tree["tokens"],
                           parents=rb.tree["parents"], n_nodes=None, n_nodes_shared=rb.N, uniforms=rb.U[:, 1:],
                           do_sample=cfg.do_sample, temperature=cfg.temperature, top_p=cfg.top_p, top_k=cfg.top_k,
                           eos_id=cfg.eos_id,
                           max_length=cfg.max_length, row_len=st.row_len, outputs=outs, dcap=rb.dcap,
                           update_len=True, active=st.active, k_layers=[st.k[l] for l in range(self.spec.n_layers)],
                           v_layers=[st.v[l] for l in range(self.spec.n_layers)], tree_hidden=rb.tree_hidden,
                           hidden_out=st.hidden, kv_rows=st.rows if isinstance(st, RoundView) else None,
                           parallel=(rb.tree["internal"], rb.tree["depths"], rb.tree["plan"], rb.drawn)
                           if rb.n_int > 0 and cfg.parallel_draws else None,
                           acc_total=rb.acc_sum, round_counter=st.round_dev)

    def view(self, st: DecodeState, B: int, n_heads: int) -> RoundView:
        """A (cached) compact view of B of st's rows; fill view.rows before
        each round run on it."""
        key = ("view", id(st), B, n_heads)
        v = self._graphs.get(key)
        if v is None:
            v = RoundView(st, B, n_heads)
            self._graphs[key] = v
        return v

    def run_round(self, st, rb: RoundBuffers, params: N.PlanParams, cfg: RoundConfig, attn_events=None,
                  phase_events=None):
        """All device work of one round, enqueued on the current stream.  st is
        a DecodeState or a RoundView (gathered before, scattered after).
        phase_events (optional): four timing events recorded at the start,
        after the proposal and tree build, after the verify forward and the
        internal-node lm_head, and after acceptance + extraction."""
        if isinstance(st, RoundView):
            st.gather()
            self._round(st, rb, params, cfg, attn_events, phase_events)
            st.scatter()
        else:
            self._round(st, rb, params, cfg, attn_events, phase_events)

    def _round(self, st, rb: RoundBuffers, params: N.PlanParams, cfg: RoundConfig, attn_events=None,
               phase_events=None):
        ev = phase_events or [None] * 4
        if ev[0] is not None:
            ev[0].record()
        if cfg.chain:
            self.propose_chain(st, rb, cfg)
            self.build_tree(st, rb, params)
            for off, n, tok in rb.chain_tokens:
                rb.tree["tokens"][:, off:off + n] = tok
        else:
            self.propose(st, rb, cfg)
            self.build_tree(st, rb, params)
        if ev[1] is not None:
            ev[1].record()
        self.verify_forward(st, rb, cfg, attn_events)
        self.accept(st, rb, cfg, phase_event=ev[2])
        if ev[3] is not None:
            ev[3].record()

    # --------------------------------------------------------------- graphs
    def graph_round(self, st: DecodeState, rb: RoundBuffers, params: N.PlanParams, cfg: RoundConfig,
                    pool=None, attn_events=None, phase_events=None) -> torch.cuda.CUDAGraph:
        """Captures run_round for this (state, buffers, plan); replay() runs it.
        attn_events / phase_events must be created with external=True to be
        captured."""
        self._attn_workspace(rb, st, cfg.attn_splits)
        if self._native_dense(cfg):
            self._prepare_linear(rb, st.B)
        M = (rb.n_heads + 1) * st.B
        if self._fused_lm_head(cfg, M):
            self._lm_head_ws(M, st.B, rb.kmax)  # allocated outside the capture
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=pool):
            self.run_round(st, rb, params, cfg, attn_events, phase_events)
        return g

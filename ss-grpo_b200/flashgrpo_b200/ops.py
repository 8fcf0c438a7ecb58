"""Torch-tensor wrappers of the C ABI (include/fg_b200.h).

Each wrapper checks devices, dtypes and layouts, then calls the entry point
on the tensor's current CUDA stream.  Nothing here computes on the host or
falls back to PyTorch kernels.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _native as N

_DTYPES = {torch.float32: N.FG_DTYPE_F32, torch.bfloat16: N.FG_DTYPE_BF16, torch.float16: N.FG_DTYPE_F16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError as exc:
        raise TypeError(f"unsupported dtype {t.dtype}") from exc


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, name: str, dtype=None, contiguous=True):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the hot path has no CPU implementation)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _out(t: torch.Tensor, name: str, dtype, n: int):
    """An output the kernel writes as n contiguous elements of dtype."""
    if t.dtype != dtype or not t.is_contiguous() or t.numel() < n:
        raise ValueError(f"{name} must be a contiguous {dtype} tensor of at least {n} elements")


def _topk_out(topk_out, rows: int, k: int):
    idx, val, mx, lse = topk_out
    _out(idx, "top-k indices", torch.int32, rows * k)
    _out(val, "top-k values", torch.float32, rows * k)
    _out(mx, "row maxima", torch.float32, rows)
    if lse is not None:
        _out(lse, "row logsumexp", torch.float32, rows)


def _rows(t: torch.Tensor, name: str) -> tuple[int, int]:
    """(row stride, vocab) of a 2-D tensor whose last dim is contiguous."""
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be 2-D with a contiguous last dimension")
    return t.stride(0), t.shape[1]


# ----------------------------------------------------------------- sampling
def philox_uniforms(seed: int, seq_ids: torch.Tensor, round_idx: int, n_draws: int,
                    out: torch.Tensor | None = None, round_dev: torch.Tensor | None = None) -> torch.Tensor:
    _need(seq_ids, "seq_ids", torch.int32)
    n = seq_ids.shape[0]
    if out is None:
        out = torch.empty((n, n_draws), dtype=torch.float32, device=seq_ids.device)
    N.call("fg_philox_uniforms", ctypes.c_uint64(seed & (2 ** 64 - 1)), _ptr(seq_ids), n, int(round_idx),
           _ptr(round_dev), int(n_draws), _ptr(out), _stream(seq_ids))
    return out


def sample_rows(logits: torch.Tensor, uniforms: torch.Tensor, *, do_sample: bool = True, temperature: float = 1.0,
                top_p: float = 1.0, top_k: int | None = None, forced: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """fg-icdf-v1 draw per row (fg-icdf-v1n when 0 < top_p < 1, fg-icdf-v1k
    when 0 < top_k < vocab); uniforms [n] or [n, k] (column 0 is used)."""
    _need(logits, "logits", contiguous=False)
    stride, vocab = _rows(logits, "logits")
    _need(uniforms, "uniforms", torch.float32, contiguous=False)
    u_stride = uniforms.stride(0) if uniforms.dim() == 2 else 1
    n = logits.shape[0]
    if forced is not None:
        _need(forced, "forced", torch.int32)
    if out is None:
        out = torch.empty(n, dtype=torch.int32, device=logits.device)
    N.call("fg_sample_rows", _ptr(logits), dtype_code(logits), stride, vocab, n, _ptr(uniforms), u_stride,
           int(bool(do_sample)), float(temperature), float(top_p), int(top_k or 0), _ptr(forced), _ptr(out),
           _stream(logits))
    return out


def row_topk(logits: torch.Tensor, k: int, out=None, *, with_lse: bool = True):
    """(idx int32 [n,k], val f32 [n,k], row max f32 [n], logsumexp f32 [n] or None)."""
    _need(logits, "logits", contiguous=False)
    stride, vocab = _rows(logits, "logits")
    n = logits.shape[0]
    dev = logits.device
    if out is None:
        out = (torch.empty((n, k), dtype=torch.int32, device=dev), torch.empty((n, k), dtype=torch.float32, device=dev),
               torch.empty(n, dtype=torch.float32, device=dev),
               torch.empty(n, dtype=torch.float32, device=dev) if with_lse else None)
    idx, val, mx, lse = out
    N.call("fg_row_topk", _ptr(logits), dtype_code(logits), stride, vocab, n, int(k), _ptr(idx), _ptr(val), _ptr(mx),
           _ptr(lse), _stream(logits))
    return out


def lm_head_topk_workspace_bytes(M: int, V: int, topk_row0: int, k: int) -> int:
    return int(N.load().fg_lm_head_topk_workspace_size(int(M), int(V), int(topk_row0), int(k)))


def lm_head_topk(x: torch.Tensor, weight: torch.Tensor, *, n_logit_rows: int, logits: torch.Tensor | None,
                 topk_row0: int, k: int, topk_out, workspace: torch.Tensor):
    """Fused lm_head + top-k (bf16): logits of rows [0, n_logit_rows) into
    `logits`, and for rows [topk_row0, M) the fg_row_topk outputs
    (idx, val, max, lse-or-None) in `topk_out`."""
    _need(x, "x", contiguous=False)
    _need(weight, "weight", contiguous=False)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise ValueError("lm_head_topk is the bf16 path")
    M, H = x.shape
    V = weight.shape[0]
    if x.stride(1) != 1 or weight.stride(1) != 1 or (logits is not None and logits.stride(1) != 1):
        raise ValueError("rows must be contiguous")
    idx, val, mx, lse = topk_out if topk_out is not None else (None, None, None, None)
    N.call("fg_lm_head_topk", _ptr(x), N.FG_DTYPE_BF16, x.stride(0), M, H, _ptr(weight), weight.stride(0), V,
           int(n_logit_rows), _ptr(logits), logits.stride(0) if logits is not None else 0, int(topk_row0), int(k),
           _ptr(idx), _ptr(val), _ptr(mx), _ptr(lse), _ptr(workspace),
           workspace.numel() * workspace.element_size() if workspace is not None else 0, _stream(x),
           n_launch=1 + (int(topk_row0) < M))
    return topk_out


def medusa_propose_workspace_bytes(B: int, H: int, V: int, n_heads: int, k: int) -> int:
    return int(N.load().fg_medusa_propose_workspace_size(int(B), int(H), int(V), int(n_heads), int(k)))


def medusa_propose(x: torch.Tensor, B: int, heads: list[dict], lm_head: torch.Tensor, *, root_logits, k: int,
                   topk_out, workspace: torch.Tensor, eps: float = 1e-5):
    """fg_medusa_propose (bf16): x [(1 + len(heads)) B, H] holds the root
    hidden states in rows [0, B); head i's projected states are written to
    rows [(i + 1) B, (i + 2) B), then the lm_head writes the root rows'
    logits to root_logits (or skips them when None) and the head rows' top-k
    to topk_out (idx, val, max, lse-or-None; rows i * B + b).  heads: dicts
    with norm_w, norm_b, fc_w, fc_b."""
    n = len(heads)
    _need(x, "x")
    _need(lm_head, "lm_head", contiguous=False)
    M, H = x.shape
    if M != (1 + n) * B:
        raise ValueError("x must have (1 + n_heads) * B rows")
    if x.dtype != torch.bfloat16 or lm_head.dtype != torch.bfloat16 or lm_head.stride(1) != 1:
        raise ValueError("medusa_propose is the bf16 path with row-contiguous weights")
    arr = (N.MedusaHead * max(n, 1))()
    for i, hw in enumerate(heads):
        for f in ("norm_w", "norm_b", "fc_w", "fc_b"):
            _need(hw[f], f)
            if hw[f].dtype != torch.bfloat16:
                raise ValueError(f"head {i} {f} must be bf16")
        if hw["fc_w"].shape != (H, H) or hw["fc_b"].shape != (H,):
            raise ValueError(f"head {i}: fc must be [H, H] with bias [H]")
        arr[i] = N.MedusaHead(_ptr(hw["norm_w"]), _ptr(hw["norm_b"]), _ptr(hw["fc_w"]), _ptr(hw["fc_b"]))
    V = lm_head.shape[0]
    if root_logits is not None and (root_logits.dtype != torch.bfloat16 or root_logits.dim() != 2
                                    or root_logits.stride(1) != 1 or root_logits.shape[0] < B
                                    or root_logits.shape[1] < V):
        raise ValueError("root_logits must be bf16 [>= B, >= V] with contiguous rows")
    if n > 0:
        if topk_out is None:
            raise ValueError("topk_out is required when there are heads")
        _topk_out(topk_out, n * B, k)
    idx, val, mx, lse = topk_out if topk_out is not None else (None, None, None, None)
    # LayerNorm and finishing pass per 8 heads, one fc GEMM per head, lm_head (+ top-k merge)
    n_launch = (2 * ((n + 7) // 8) + n if n > 0 else 0) + 1 + (n > 0)
    N.call("fg_medusa_propose", _ptr(x), N.FG_DTYPE_BF16, int(B), H, arr, n, float(eps), _ptr(lm_head),
           lm_head.stride(0), lm_head.shape[0], _ptr(root_logits),
           root_logits.stride(0) if root_logits is not None else 0, int(k), _ptr(idx), _ptr(val), _ptr(mx),
           _ptr(lse), _ptr(workspace), workspace.numel() * workspace.element_size() if workspace is not None else 0,
           _stream(x), n_launch=n_launch)
    return topk_out


def chain_step_workspace_bytes(M: int, H: int, bottleneck: int, V: int, k: int) -> int:
    return int(N.load().fg_chain_step_workspace_size(int(M), int(H), int(bottleneck), int(V), int(k)))


def chain_step(state: torch.Tensor, tokens: torch.Tensor, *, n_parent: int, fanout: int, n_child: int,
               embed: torch.Tensor, cell: dict, lm_head: torch.Tensor | None, k: int, state_out: torch.Tensor,
               topk_out, workspace: torch.Tensor, eps: float = 1e-5):
    """fg_chain_step (bf16): state [n_seq * n_parent, H]; tokens [n_seq, >=
    n_child] int32 (row b's children's tokens, any row stride); cell: the
    chain_cell.* tensors by their state-dict names.  Writes the n_seq *
    n_child new states to state_out and, when k > 0, their lm_head top-k to
    topk_out (idx, val, max, lse-or-None)."""
    _need(state, "state")
    _need(state_out, "state_out")
    _need(embed, "embed", contiguous=False)
    _need(tokens, "tokens", dtype=torch.int32, contiguous=False)
    if tokens.dim() != 2 or tokens.stride(1) != 1 or embed.stride(1) != 1:
        raise ValueError("tokens and embed need contiguous rows")
    for t in (state, state_out, embed):
        if t.dtype != torch.bfloat16:
            raise ValueError("chain_step is the bf16 path")
    H = state.shape[1]
    n_seq = tokens.shape[0]
    names = ("state_norm.weight", "state_norm.bias", "token_norm.weight", "token_norm.bias", "state_proj.weight",
             "token_proj.weight", "out_proj.weight", "out_proj.bias", "gate")
    for nm in names:
        _need(cell[nm], nm)
        if cell[nm].dtype != torch.bfloat16:
            raise ValueError(f"chain cell {nm} must be bf16")
    bn = cell["state_proj.weight"].shape[0]
    c = N.ChainCell(*[_ptr(cell[nm]) for nm in names], int(bn))
    V = lm_head.shape[0] if lm_head is not None else embed.shape[0]
    if embed.shape[0] < V:
        raise ValueError("the embedding table needs the lm_head's V rows (tokens are checked against V)")
    if state.shape[0] != n_seq * n_parent or tokens.shape[1] < n_child:
        raise ValueError("state must have n_seq * n_parent rows and tokens n_child columns")
    _out(state_out, "state_out", torch.bfloat16, n_seq * n_child * H)
    if k > 0:
        if topk_out is None or lm_head is None:
            raise ValueError("k > 0 needs lm_head and topk_out")
        _topk_out(topk_out, n_seq * n_child, k)
    idx, val, mx, lse = topk_out if topk_out is not None else (None, None, None, None)
    M = n_seq * n_child
    # per pass of 256 rows: norms, 3 projections, mix, finish (+ lm_head and its top-k merge)
    n_launch = (M + 255) // 256 * (6 + (2 if k > 0 else 0))
    N.call("fg_chain_step", _ptr(state), _ptr(tokens), tokens.stride(0), n_seq, int(n_parent), int(fanout),
           int(n_child), _ptr(embed), embed.stride(0), H, N.FG_DTYPE_BF16, ctypes.byref(c), float(eps),
           _ptr(state_out), _ptr(lm_head), lm_head.stride(0) if lm_head is not None else 0, V, int(k), _ptr(idx), _ptr(val), _ptr(mx),
           _ptr(lse), _ptr(workspace), workspace.numel() * workspace.element_size(), _stream(state),
           n_launch=n_launch)
    return state_out


# ---------------------------------------------------------------- planning
def plan_params(*, tree_mode: str, active_batch_size: int, num_medusa_heads: int, cpeak_nodes: int,
                min_tree_nodes_per_seq: int, max_tree_nodes_per_seq: int, max_tree_depth: int,
                fixed_tree_topk_by_depth, adaptive_tree_enabled: bool = False, adaptive_min_topk_by_depth=(1, 1, 1),
                adaptive_confidence_metric: str = "top1_prob", adaptive_confidence_quantile: float = 0.25,
                adaptive_confidence_low: float = 0.15, adaptive_confidence_high: float = 0.45,
                adaptive_depth_weight_decay: float = 0.5) -> N.PlanParams:
    modes = {"fixed": 0, "concurrency_aware": 1, "explicit": 2}
    if tree_mode not in modes:
        raise ValueError(f"Unsupported tree_mode={tree_mode}")
    p = N.PlanParams()
    p.tree_mode = modes[tree_mode]
    p.active_batch_size = int(active_batch_size)
    p.num_medusa_heads = int(num_medusa_heads)
    p.cpeak_nodes = int(cpeak_nodes)
    p.min_tree_nodes_per_seq = int(min_tree_nodes_per_seq)
    p.max_tree_nodes_per_seq = int(max_tree_nodes_per_seq)
    p.max_tree_depth = int(max_tree_depth)
    fixed = [int(k) for k in fixed_tree_topk_by_depth][: N.FG_MAX_DEPTHS]
    p.n_fixed = len(fixed)
    for i, k in enumerate(fixed):
        p.fixed_topk[i] = k
    p.adaptive = int(bool(adaptive_tree_enabled))
    mins = [int(k) for k in adaptive_min_topk_by_depth][: N.FG_MAX_DEPTHS]
    p.n_min = len(mins)
    for i, k in enumerate(mins):
        p.adaptive_min_topk[i] = k
    if adaptive_confidence_metric not in ("top1_prob", "margin"):
        raise ValueError(f"unknown adaptive_confidence_metric {adaptive_confidence_metric}")
    p.confidence_metric = 1 if adaptive_confidence_metric == "margin" else 0
    p.confidence_quantile = float(adaptive_confidence_quantile)
    p.confidence_low = float(adaptive_confidence_low)
    p.confidence_high = float(adaptive_confidence_high)
    w = max(float(adaptive_depth_weight_decay), 1e-3)
    for d in range(N.FG_MAX_DEPTHS):
        p.depth_weight[d] = w ** d
    p.log_gain[0] = 0.0
    for v in range(1, 65):
        p.log_gain[v] = math.log1p(v) - math.log(v)
    return p


def build_tree(params: N.PlanParams, root: torch.Tensor, cand_idx: torch.Tensor | None, cand_val, head_max,
               head_lse, *, nmax: int, logits_dtype: torch.dtype, row_len: torch.Tensor, out: dict | None = None):
    """K2.  cand_* are [n_heads, B, kmax]; returns a dict of device tensors."""
    _need(root, "root", torch.int32)
    _need(row_len, "row_len", torch.int32)
    B = root.shape[0]
    dev = root.device
    if cand_idx is not None:
        _need(cand_idx, "cand_idx", torch.int32)
        n_heads, _, kmax = cand_idx.shape
    else:
        n_heads, kmax = 0, 1
    if out is None:
        i32 = dict(dtype=torch.int32, device=dev)
        out = {"tokens": torch.empty((B, nmax), **i32), "positions": torch.empty((B, nmax), **i32),
               "slot": torch.empty((B, nmax), **i32), "parents": torch.empty(nmax, **i32),
               "depths": torch.empty(nmax, **i32), "anc": torch.empty((nmax, 4), **i32),
               "internal": torch.empty(nmax, **i32), "plan": torch.empty(16, **i32)}
    N.call("fg_build_tree", ctypes.byref(params), _ptr(root), _ptr(cand_idx), _ptr(cand_val), _ptr(head_max),
           _ptr(head_lse), n_heads, kmax, B, nmax, _DTYPES[logits_dtype], _ptr(row_len), _ptr(out["tokens"]),
           _ptr(out["positions"]), _ptr(out["slot"]), _ptr(out["parents"]), _ptr(out["depths"]), _ptr(out["anc"]),
           _ptr(out["internal"]), _ptr(out["plan"]), _stream(root))
    return out


# --------------------------------------------------------------- attention
def kv_layer(k: torch.Tensor, v: torch.Tensor, rows: torch.Tensor | None = None) -> N.KvLayer:
    """fg_kv_layer of caches [batch, Hkv, capacity, D]; rows (int32 [B],
    optional): call row b reads / writes cache row rows[b]."""
    if k.shape != v.shape or k.stride() != v.stride() or k.dim() != 4 or k.stride(3) != 1:
        raise ValueError("K and V caches must be [B, Hkv, capacity, D] views with identical strides")
    if rows is not None:
        _need(rows, "rows", torch.int32)
    return N.KvLayer(k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k.stride(2), k.shape[2],
                     _ptr(rows), k.shape[0] if rows is not None else 0)


def attention_workspace_bytes(B, n_nodes, n_q_heads, n_kv_heads, head_dim, *, num_splits=0, max_kv_len=0) -> int:
    return int(N.load().fg_tree_attention_workspace_size(B, n_nodes, n_q_heads, n_kv_heads, head_dim, num_splits,
                                                         max_kv_len))


def tree_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, kv_len: torch.Tensor,
                   anc: torch.Tensor, *, scale: float, out: torch.Tensor | None = None,
                   workspace: torch.Tensor | None = None, num_splits: int = 0, max_kv_len: int = 0,
                   kv: N.KvLayer | None = None) -> torch.Tensor:
    """K3.  q [B, N, Hq, D]; caches [B, Hkv, cap, D]; anc int32 [N, 4] bits."""
    _need(q, "q")
    _need(kv_len, "kv_len", torch.int32)
    _need(anc, "anc", torch.int32)
    B, n_nodes, hq, D = q.shape
    hkv = k_cache.shape[1]
    if out is None:
        out = torch.empty_like(q)
    if kv is None:
        kv = kv_layer(k_cache, v_cache)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    N.call("fg_tree_attention", _ptr(q), dtype_code(q), ctypes.byref(kv), _ptr(kv_len), _ptr(anc), B, n_nodes, hq,
           hkv, D, float(scale), _ptr(out), _ptr(workspace), ws_bytes, int(num_splits), int(max_kv_len), _stream(q))
    return out


# ------------------------------------------------------ accept + extraction
def layer_pointer_arrays(k_layers, v_layers):
    n = len(k_layers)
    kp = (ctypes.c_uint64 * max(n, 1))(*[t.data_ptr() for t in k_layers])
    vp = (ctypes.c_uint64 * max(n, 1))(*[t.data_ptr() for t in v_layers])
    return kp, vp


def accept_extract(*, logits, slot, tokens, parents, n_nodes, uniforms, do_sample, temperature, eos_id, max_length,
                   row_len, outputs: dict, dcap: int, update_len: bool = True, active=None, k_layers=(), v_layers=(),
                   tree_hidden=None, hidden_out=None, parents_shared: bool = True, n_nodes_shared: int = 0,
                   top_p: float = 1.0, top_k: int | None = None, kv_rows=None, parallel=None, acc_total=None,
                   round_counter=None):
    """K4.  outputs holds int32 tensors acc_tokens/acc_nodes [B, dcap] and
    acc_len/correction/pending/last_node/finished [B]; kv_rows (int32 [B],
    optional): row b compacts cache row kv_rows[b] of k_layers/v_layers.
    parallel (optional, shared topology): (internal [nmax], depths [nmax],
    plan_out [16] or None, drawn int32 [logits rows]) -- every internal
    node's draw in parallel before the walk (the same tokens).  acc_total
    (int64 [1]) and round_counter (int32 [1]), optional: the round's
    accepted tokens are added to the first, 1 to the second."""
    _need(logits, "logits", contiguous=False)
    stride, vocab = _rows(logits, "logits")
    for name, t in (("slot", slot), ("tokens", tokens), ("parents", parents), ("row_len", row_len)):
        _need(t, name, torch.int32)
    _need(uniforms, "uniforms", torch.float32, contiguous=False)
    if uniforms.dim() != 2 or uniforms.stride(1) != 1:
        raise ValueError("uniforms must be [B, draws] with contiguous rows")
    B, nmax = tokens.shape
    a = N.AcceptArgs()
    a.logits, a.logits_dtype, a.logits_row_stride, a.vocab = logits.data_ptr(), dtype_code(logits), stride, vocab
    a.slot, a.tokens, a.parents = slot.data_ptr(), tokens.data_ptr(), parents.data_ptr()
    a.parent_stride = 0 if parents_shared else nmax
    a.n_nodes = _ptr(n_nodes)
    a.n_nodes_shared = int(n_nodes_shared)
    a.nmax = nmax
    a.uniforms, a.u_stride = uniforms.data_ptr(), uniforms.stride(0)
    a.B, a.do_sample, a.temperature, a.top_p = B, int(bool(do_sample)), float(temperature), float(top_p)
    a.top_k = int(top_k or 0)
    a.eos_id, a.max_length = int(eos_id), int(max_length)
    a.row_len, a.update_len, a.active, a.dcap = row_len.data_ptr(), int(bool(update_len)), _ptr(active), int(dcap)
    for key in ("acc_tokens", "acc_nodes", "acc_len", "correction", "pending", "last_node", "finished"):
        setattr(a, key, outputs[key].data_ptr())
    kp = vp = None
    if k_layers:
        ref = k_layers[0]
        kp, vp = layer_pointer_arrays(k_layers, v_layers)
        a.n_layers = len(k_layers)
        a.k_layers, a.v_layers = kp, vp
        a.kv_elem_bytes, a.n_kv_heads, a.head_dim = ref.element_size(), ref.shape[1], ref.shape[3]
        a.kv_stride_b, a.kv_stride_h, a.kv_stride_s = ref.stride(0), ref.stride(1), ref.stride(2)
        if kv_rows is not None:
            _need(kv_rows, "kv_rows", torch.int32)
            a.kv_rows, a.kv_batch = kv_rows.data_ptr(), ref.shape[0]
    if hidden_out is not None:
        a.tree_hidden, a.hidden_out = tree_hidden.data_ptr(), hidden_out.data_ptr()
        a.hidden_dim, a.hidden_elem_bytes = hidden_out.shape[-1], hidden_out.element_size()
    if acc_total is not None:
        _need(acc_total, "acc_total", torch.int64)
        a.acc_total = acc_total.data_ptr()
    if round_counter is not None:
        _need(round_counter, "round_counter", torch.int32)
        a.round_counter = round_counter.data_ptr()
    n_launch = 1
    if parallel is not None:
        internal, depths, plan_out, drawn = parallel
        for name, t in (("internal", internal), ("depths", depths), ("drawn", drawn)):
            _need(t, name, torch.int32)
        if drawn.numel() < logits.shape[0]:
            raise ValueError("drawn needs one entry per logits row")
        a.internal, a.depths, a.plan_out = internal.data_ptr(), depths.data_ptr(), _ptr(plan_out)
        a.internal_rows, a.drawn = logits.shape[0], drawn.data_ptr()
        n_launch = 2
    N.call("fg_accept_extract", ctypes.byref(a), _stream(tokens), n_launch=n_launch)
    return outputs


def extract_path(k_layers, v_layers, row_len, acc_nodes, acc_len) -> None:
    """In-place compaction of accepted slots for caches [B, Hkv, S, D]."""
    ref = k_layers[0]
    kp, vp = layer_pointer_arrays(k_layers, v_layers)
    N.call("fg_extract_path", len(k_layers), kp, vp, ref.element_size(), ref.shape[0], ref.shape[1], ref.shape[3],
           ref.stride(0), ref.stride(1), ref.stride(2), _ptr(row_len), _ptr(acc_nodes), _ptr(acc_len),
           acc_nodes.shape[1], _stream(ref))


# ------------------------------------------------------------- layer pieces
def rope_table(positions, inv_freq, attention_scaling, dtype, out=None):
    """[2, n_tokens, head_dim / 2] cos/sin in `dtype` for fg_rope_kv_write."""
    _need(positions, "positions", torch.int32)
    n, half = positions.numel(), inv_freq.numel()
    if out is None:
        out = torch.empty((2, n, half), dtype=dtype, device=positions.device)
    N.call("fg_rope_table", _ptr(positions), n, _ptr(inv_freq), half, float(attention_scaling),
           _DTYPES[dtype], _ptr(out), _stream(positions))
    return out


def rope_kv_write(qkv, positions, inv_freq, attention_scaling, *, B, n_nodes, n_q_heads, n_kv_heads, head_dim,
                  kv_len, k_cache, v_cache, q_out, kv: N.KvLayer | None = None, cos_sin=None):
    if kv is None:
        kv = kv_layer(k_cache, v_cache)
    N.call("fg_rope_kv_write", _ptr(qkv), dtype_code(qkv), _ptr(positions), _ptr(inv_freq), float(attention_scaling),
           B, n_nodes, n_q_heads, n_kv_heads, head_dim, _ptr(kv_len), ctypes.byref(kv), _ptr(q_out), _ptr(cos_sin),
           _stream(qkv))
    return q_out


def rmsnorm(x, weight, eps, out=None):
    out = torch.empty_like(x) if out is None else out
    N.call("fg_rmsnorm", _ptr(x), _ptr(weight), dtype_code(x), x.numel() // x.shape[-1], x.shape[-1], float(eps),
           _ptr(out), _stream(x))
    return out


def layernorm(x, weight, bias, eps, out=None):
    out = torch.empty_like(x) if out is None else out
    N.call("fg_layernorm", _ptr(x), _ptr(weight), _ptr(bias), dtype_code(x), x.numel() // x.shape[-1], x.shape[-1],
           float(eps), _ptr(out), _stream(x))
    return out


def gate_up_silu(x: torch.Tensor, w_gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fg_gate_up_silu (bf16): silu(x @ w_gate_up[:I].T) * (x @ w_gate_up[I:].T)
    with the GEMM and the gating in one tcgen05 kernel; x [T, H], w_gate_up
    [2I, H]; returns act [T, I]."""
    _need(x, "x")
    _need(w_gate_up, "w_gate_up")
    if x.dtype != torch.bfloat16 or w_gate_up.dtype != torch.bfloat16:
        raise ValueError("gate_up_silu is the bf16 path")
    T, H = x.shape
    I = w_gate_up.shape[0] // 2
    if w_gate_up.shape != (2 * I, H):
        raise ValueError("w_gate_up must be [2I, H]")
    if out is None:
        out = torch.empty((T, I), dtype=x.dtype, device=x.device)
    _need(out, "out")
    if out.shape != (T, I) or out.dtype != torch.bfloat16:
        raise ValueError("out must be bf16 [T, I]")
    N.call("fg_gate_up_silu", _ptr(x), N.FG_DTYPE_BF16, T, H, _ptr(w_gate_up), I, _ptr(out), _stream(x))
    return out


EPI_STORE, EPI_RESID, EPI_SWIGLU = 0, 1, 2


def linear_workspace_bytes(M: int, N_out: int, K: int, epilogue: int = EPI_STORE, bn: int = 0, splits: int = 0,
                           bm: int = 0) -> int:
    return int(N.load().fg_linear_workspace_size(M, N_out, K, epilogue, bm, bn, splits))


def _row_stride(t: torch.Tensor, name: str):
    """A 2-D bf16 CUDA tensor with contiguous rows; returns its row stride."""
    _need(t, name, torch.bfloat16, contiguous=False)
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be 2-D with contiguous rows")
    return t.stride(0)


def linear(x: torch.Tensor, w: torch.Tensor, *, bias: torch.Tensor | None = None, resid: torch.Tensor | None = None,
           out: torch.Tensor | None = None, epilogue: int | None = None, bn: int = 0, splits: int = 0,
           bm: int = 0, stages: int = 0, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """fg_linear (bf16, tcgen05): out = x @ w.T + bias (EPI_STORE), resid +
    x @ w.T + bias (EPI_RESID, the default when resid is given; resid may be
    out), or the SwiGLU of the gate rows w[:I] and up rows w[I:] (EPI_SWIGLU).
    x [M, K], w [N, K] (or [2I, K]); tile tokens bm (128 / 256), outputs bn,
    k ranges `splits` and ring `stages`, 0 = chosen by the library; split-K
    tiles need `workspace` (linear_workspace_bytes, zero-filled once)."""
    if epilogue is None:
        epilogue = EPI_RESID if resid is not None else EPI_STORE
    ldx = _row_stride(x, "x")
    ldw = _row_stride(w, "w")
    M, K = x.shape
    if ldx != K or ldw != K or w.shape[1] != K:
        raise ValueError("x and w need densely packed rows of the same K")
    n_out = w.shape[0] // 2 if epilogue == EPI_SWIGLU else w.shape[0]
    if out is None:
        out = torch.empty((M, n_out), dtype=x.dtype, device=x.device)
    ldo = _row_stride(out, "out")
    if out.shape != (M, n_out):
        raise ValueError(f"out must be [{M}, {n_out}]")
    ldr = 0
    if resid is not None:
        ldr = _row_stride(resid, "resid")
        if resid.shape != (M, n_out):
            raise ValueError("resid must have out's shape")
    if bias is not None:
        _need(bias, "bias", torch.bfloat16)
        if bias.shape != (n_out,):
            raise ValueError("bias must be [N]")
    need = linear_workspace_bytes(M, n_out, K, epilogue, bn, splits, bm)
    if need:
        if workspace is None or workspace.numel() * workspace.element_size() < need:
            raise ValueError(f"this tiling needs a zero-filled workspace of {need} bytes")
        _need(workspace, "workspace", contiguous=True)
    N.call("fg_linear", _ptr(x), N.FG_DTYPE_BF16, M, K, _ptr(w), n_out, _ptr(bias), _ptr(resid), ldr, _ptr(out), ldo,
           epilogue, bm, bn, splits, stages, _ptr(workspace) if need else None, need, _stream(x))
    return out


def silu_mul(gu, out=None):
    inter = gu.shape[-1] // 2
    rows = gu.numel() // gu.shape[-1]
    if out is None:
        out = torch.empty((*gu.shape[:-1], inter), dtype=gu.dtype, device=gu.device)
    N.call("fg_silu_mul", _ptr(gu), dtype_code(gu), rows, inter, _ptr(out), _stream(gu))
    return out


def silu_residual(x, y, out=None):
    out = torch.empty_like(x) if out is None else out
    N.call("fg_silu_residual", _ptr(x), _ptr(y), dtype_code(x), x.numel(), _ptr(out), _stream(x))
    return out


def gather_rows(src: torch.Tensor, idx: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[r] = src[idx[r]] along dim 0 (rows contiguous)."""
    row_bytes = src[0].numel() * src.element_size()
    if out is None:
        out = torch.empty((idx.shape[0], *src.shape[1:]), dtype=src.dtype, device=src.device)
    N.call("fg_gather_rows", _ptr(src), src.stride(0) * src.element_size(), _ptr(idx), idx.shape[0], row_bytes,
           _ptr(out), out.stride(0) * out.element_size(), _stream(src))
    return out

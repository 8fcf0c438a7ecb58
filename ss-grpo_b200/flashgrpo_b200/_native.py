"""ctypes binding of libfgb200.so, the C ABI declared in include/fg_b200.h.

The library is the only compute path: if it is missing or fails to load, the
import of any op raises -- there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("FG_B200_LIB", _PKG / "libfgb200.so"))

FG_OK, FG_EINVAL, FG_ECAPACITY, FG_ETIMEOUT, FG_ECUDA, FG_EUNSUPPORTED = range(6)
FG_DTYPE_F32, FG_DTYPE_BF16, FG_DTYPE_F16 = 0, 1, 2
FG_MAX_TREE_NODES = 128
FG_MAX_DEPTHS = 8
FG_MAX_TOPK = 16
FG_MAX_PATH = 16
FG_MAX_LAYERS = 128
FG_NOALLOC_SCRATCH_BYTES = 32 << 20

c_i32, c_i64, c_f32, c_f64, c_u64, c_vp = (ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_double,
                                          ctypes.c_uint64, ctypes.c_void_p)


class PlanParams(ctypes.Structure):
    _fields_ = [
        ("tree_mode", c_i32), ("active_batch_size", c_i32), ("num_medusa_heads", c_i32), ("cpeak_nodes", c_i32),
        ("min_tree_nodes_per_seq", c_i32), ("max_tree_nodes_per_seq", c_i32), ("max_tree_depth", c_i32),
        ("n_fixed", c_i32), ("fixed_topk", c_i32 * FG_MAX_DEPTHS), ("adaptive", c_i32), ("n_min", c_i32),
        ("adaptive_min_topk", c_i32 * FG_MAX_DEPTHS), ("confidence_metric", c_i32), ("confidence_quantile", c_f32),
        ("confidence_low", c_f64), ("confidence_high", c_f64), ("depth_weight", c_f64 * FG_MAX_DEPTHS),
        ("log_gain", c_f64 * 65),
    ]


class KvLayer(ctypes.Structure):
    _fields_ = [("k", c_vp), ("v", c_vp), ("stride_b", c_i64), ("stride_h", c_i64), ("stride_s", c_i64),
                ("capacity", c_i32), ("rows", c_vp), ("batch", c_i32)]


class MedusaHead(ctypes.Structure):
    _fields_ = [("norm_w", c_vp), ("norm_b", c_vp), ("fc_w", c_vp), ("fc_b", c_vp)]


class ChainCell(ctypes.Structure):
    _fields_ = [("state_norm_w", c_vp), ("state_norm_b", c_vp), ("token_norm_w", c_vp), ("token_norm_b", c_vp),
                ("state_proj_w", c_vp), ("token_proj_w", c_vp), ("out_proj_w", c_vp), ("out_proj_b", c_vp),
                ("gate", c_vp), ("bottleneck", c_i32)]


class AcceptArgs(ctypes.Structure):
    _fields_ = [
        ("logits", c_vp), ("logits_dtype", c_i32), ("logits_row_stride", c_i64), ("vocab", c_i32),
        ("slot", c_vp), ("tokens", c_vp), ("parents", c_vp), ("parent_stride", c_i32), ("n_nodes", c_vp),
        ("n_nodes_shared", c_i32), ("nmax", c_i32), ("uniforms", c_vp), ("u_stride", c_i32), ("B", c_i32),
        ("do_sample", c_i32), ("temperature", c_f32), ("top_p", c_f32), ("top_k", c_i32), ("eos_id", c_i32), ("max_length", c_i32), ("row_len", c_vp),
        ("update_len", c_i32), ("active", c_vp), ("dcap", c_i32), ("acc_tokens", c_vp), ("acc_nodes", c_vp),
        ("acc_len", c_vp), ("correction", c_vp), ("pending", c_vp), ("last_node", c_vp), ("finished", c_vp),
        ("n_layers", c_i32), ("k_layers", ctypes.POINTER(c_u64)), ("v_layers", ctypes.POINTER(c_u64)),
        ("kv_elem_bytes", c_i32), ("n_kv_heads", c_i32), ("head_dim", c_i32), ("kv_stride_b", c_i64),
        ("kv_stride_h", c_i64), ("kv_stride_s", c_i64), ("tree_hidden", c_vp), ("hidden_out", c_vp),
        ("hidden_dim", c_i32), ("hidden_elem_bytes", c_i32), ("kv_rows", c_vp), ("kv_batch", c_i32),
        ("internal", c_vp), ("depths", c_vp), ("plan_out", c_vp), ("internal_rows", c_i32), ("drawn", c_vp),
        ("acc_total", c_vp), ("round_counter", c_vp),
    ]


# name -> (restype, argtypes); every symbol declared in include/fg_b200.h
SIGNATURES = {
    "fg_version": (ctypes.c_char_p, []),
    "fg_status_string": (ctypes.c_char_p, [c_i32]),
    "fg_last_cuda_error": (c_i32, []),
    "fg_read_device_error": (c_i32, [ctypes.POINTER(c_i32), c_i32]),
    "fg_wait_flag": (c_i32, [c_vp, c_i64, c_vp, c_vp]),
    "fg_philox_uniforms": (c_i32, [c_u64, c_vp, c_i32, c_i32, c_vp, c_i32, c_vp, c_vp]),
    "fg_sample_rows": (c_i32, [c_vp, c_i32, c_i64, c_i32, c_i32, c_vp, c_i64, c_i32, c_f32, c_f32, c_i32, c_vp,
                               c_vp, c_vp]),
    "fg_row_topk": (c_i32, [c_vp, c_i32, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "fg_lm_head_topk_workspace_size": (ctypes.c_size_t, [c_i32, c_i32, c_i32, c_i32]),
    "fg_lm_head_topk": (c_i32, [c_vp, c_i32, c_i64, c_i32, c_i32, c_vp, c_i64, c_i32, c_i32, c_vp, c_i64, c_i32, c_i32,
                                c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_size_t, c_vp]),
    "fg_medusa_propose_workspace_size": (ctypes.c_size_t, [c_i32, c_i32, c_i32, c_i32, c_i32]),
    "fg_medusa_propose": (c_i32, [c_vp, c_i32, c_i32, c_i32, ctypes.POINTER(MedusaHead), c_i32, c_f32, c_vp, c_i64,
                                  c_i32, c_vp, c_i64, c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_size_t, c_vp]),
    "fg_chain_step_workspace_size": (ctypes.c_size_t, [c_i32, c_i32, c_i32, c_i32, c_i32]),
    "fg_chain_step": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_vp, c_i64, c_i32, c_i32,
                              ctypes.POINTER(ChainCell), c_f32, c_vp, c_vp, c_i64, c_i32, c_i32, c_vp, c_vp, c_vp,
                              c_vp, c_vp, ctypes.c_size_t, c_vp]),
    "fg_gate_up_silu": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_vp, c_i32, c_vp, c_vp]),
    "fg_linear_workspace_size": (ctypes.c_size_t, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32]),
    "fg_linear": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_vp, c_i32, c_vp, c_vp, c_i64, c_vp, c_i64, c_i32, c_i32, c_i32,
                          c_i32, c_i32, c_vp, ctypes.c_size_t, c_vp]),
    "fg_build_tree": (c_i32, [ctypes.POINTER(PlanParams), c_vp, c_vp, c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32,
                              c_i32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "fg_tree_attention_workspace_size": (ctypes.c_size_t, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32]),
    "fg_tree_attention": (c_i32, [c_vp, c_i32, ctypes.POINTER(KvLayer), c_vp, c_vp, c_i32, c_i32, c_i32, c_i32,
                                  c_i32, c_f32, c_vp, c_vp, ctypes.c_size_t, c_i32, c_i32, c_vp]),
    "fg_tree_attention_noalloc": (c_i32, [c_vp, c_i32, ctypes.POINTER(KvLayer), c_vp, c_vp, c_i32, c_i32, c_i32,
                                          c_i32, c_i32, c_f32, c_vp, c_i32, c_i32, c_vp]),
    "fg_accept_extract": (c_i32, [ctypes.POINTER(AcceptArgs), c_vp]),
    "fg_extract_path": (c_i32, [c_i32, ctypes.POINTER(c_u64), ctypes.POINTER(c_u64), c_i32, c_i32, c_i32, c_i32,
                                c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_i32, c_vp]),
    "fg_rope_kv_write": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_f32, c_i32, c_i32, c_i32, c_i32, c_i32, c_vp,
                                 ctypes.POINTER(KvLayer), c_vp, c_vp, c_vp]),
    "fg_rope_table": (c_i32, [c_vp, c_i32, c_vp, c_i32, c_f32, c_i32, c_vp, c_vp]),
    "fg_rmsnorm": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_i32, c_f32, c_vp, c_vp]),
    "fg_layernorm": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_f32, c_vp, c_vp]),
    "fg_silu_mul": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_vp, c_vp]),
    "fg_silu_residual": (c_i32, [c_vp, c_vp, c_i32, c_i64, c_vp, c_vp]),
    "fg_gather_rows": (c_i32, [c_vp, c_i64, c_vp, c_i32, c_i64, c_vp, c_i64, c_vp]),
}

_lib = None


class NativeError(RuntimeError):
    def __init__(self, fn: str, status: int):
        lib = load()
        msg = lib.fg_status_string(status).decode()
        extra = f" (cudaError {lib.fg_last_cuda_error()})" if status == FG_ECUDA else ""
        super().__init__(f"{fn} failed: {msg}{extra}")
        self.status = status


def load():
    """Loads libfgb200.so; raises if it is missing (no fallback exists)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python ss-grpo_b200/flashgrpo_b200/_build.py` "
                "(nvcc, sm_100a). There is no CPU fallback for the B200 hot path.")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


# Entry points that enqueue kernels; `launches` counts them so a caller can
# report how many of this library's kernels a step runs (one per call unless
# the caller passes the call's own count, e.g. the lm_head's top-k merge).
LAUNCHING = {"fg_wait_flag", "fg_philox_uniforms", "fg_sample_rows", "fg_row_topk", "fg_lm_head_topk", "fg_build_tree", "fg_rope_table",
             "fg_tree_attention", "fg_tree_attention_noalloc", "fg_accept_extract", "fg_extract_path", "fg_rope_kv_write", "fg_rmsnorm",
             "fg_layernorm", "fg_silu_mul", "fg_silu_residual", "fg_gather_rows", "fg_medusa_propose",
             "fg_chain_step", "fg_gate_up_silu", "fg_linear"}
launches = 0


def call(name: str, *args, n_launch: int | None = None) -> None:
    global launches
    status = getattr(load(), name)(*args)
    if status != FG_OK:
        raise NativeError(name, status)
    if name in LAUNCHING:
        launches += 1 if n_launch is None else n_launch


def read_device_error(clear: bool = True) -> int:
    out = c_i32(0)
    call("fg_read_device_error", ctypes.byref(out), int(bool(clear)))
    return int(out.value)

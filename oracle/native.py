"""ctypes bindings of the C oracle (``oracle/fg_oracle.c``).

TEST INFRASTRUCTURE ONLY -- the checker for the CUDA kernels, never the thing
measured or shipped.  Every function takes and returns numpy arrays.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libfg_oracle.so"
_lib = None

_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)
_u32p = ctypes.POINTER(ctypes.c_uint32)


def build() -> Path:
    subprocess.run(["bash", str(_HERE / "build_oracle.sh")], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(_LIB_PATH))
        _lib.fgo_exp.restype = ctypes.c_float
        _lib.fgo_exp.argtypes = [ctypes.c_float]
        _lib.fgo_uniform.restype = ctypes.c_float
        _lib.fgo_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]
        _lib.fgo_philox4x32_10.argtypes = [_u32p, _u32p, _u32p]
        _lib.fgo_philox_uniforms.argtypes = [ctypes.c_uint64, _i32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _f32p]
        _lib.fgo_chunk_len.restype = ctypes.c_int32
        _lib.fgo_chunk_len.argtypes = [ctypes.c_int32]
        _lib.fgo_sample_row.restype = ctypes.c_int32
        _lib.fgo_sample_row.argtypes = [_f32p, ctypes.c_int32, ctypes.c_float, ctypes.c_int32, ctypes.c_float]
        _lib.fgo_sample_rows.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, _f32p,
                                         ctypes.c_int32, ctypes.c_float, ctypes.c_float, ctypes.c_int32, _i32p]
        _lib.fgo_kept_set.restype = ctypes.c_int32
        _lib.fgo_kept_set.argtypes = [_f32p, ctypes.c_int32, ctypes.c_float, ctypes.c_float, ctypes.c_int32,
                                      ctypes.POINTER(ctypes.c_uint8)]
        _lib.fgo_nucleus_kept.restype = ctypes.c_int32
        _lib.fgo_nucleus_kept.argtypes = [_f32p, ctypes.c_int32, ctypes.c_float, ctypes.c_float,
                                          ctypes.POINTER(ctypes.c_uint8)]
        _lib.fgo_accept_walk.restype = ctypes.c_int32
        _lib.fgo_accept_walk.argtypes = [
            _f32p, ctypes.c_int64, ctypes.c_int32, _i32p, _i32p, _i32p, _i32p, ctypes.c_int32,
            _f32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_float, ctypes.c_float, ctypes.c_int32,
            ctypes.c_int32, ctypes.c_int32, _i32p, ctypes.c_int32, _i32p, _i32p, _i32p, _i32p, _i32p, _i32p, _i32p, _i32p,
        ]
        _lib.fgo_extract_path.argtypes = [
            ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32, ctypes.c_int32,
            ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
            _i32p, _i32p, _i32p, ctypes.c_int32,
        ]
        _lib.fgo_topk_stable.argtypes = [_f32p, ctypes.c_int32, ctypes.c_int32, _i32p, _f32p]
        _lib.fgo_build_dense_trees.argtypes = [
            _i32p, _i32p, ctypes.c_int32, _i32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
            _i32p, _i32p, _i32p, _i32p,
        ]
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def _c32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def _cf(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def fg_exp(x: float) -> float:
    return float(lib().fgo_exp(ctypes.c_float(x)))


def exp_array(x: np.ndarray) -> np.ndarray:
    f = lib().fgo_exp
    return np.array([f(float(v)) for v in np.asarray(x, dtype=np.float32).ravel()], dtype=np.float32).reshape(np.shape(x))


def philox4x32_10(ctr, key) -> list[int]:
    c = np.ascontiguousarray(ctr, dtype=np.uint32)
    k = np.ascontiguousarray(key, dtype=np.uint32)
    out = np.zeros(4, dtype=np.uint32)
    lib().fgo_philox4x32_10(_p(c, _u32p), _p(k, _u32p), _p(out, _u32p))
    return [int(v) for v in out]


def uniform(seed: int, seq_id: int, round_idx: int, draw: int) -> float:
    return float(lib().fgo_uniform(seed, seq_id, round_idx, draw))


def philox_uniforms(seed: int, seq_ids, round_idx: int, n_draws: int) -> np.ndarray:
    s = _c32(seq_ids)
    out = np.zeros((len(s), n_draws), dtype=np.float32)
    lib().fgo_philox_uniforms(seed, _p(s, _i32p), len(s), round_idx, n_draws, _p(out, _f32p))
    return out


def chunk_len(V: int) -> int:
    return int(lib().fgo_chunk_len(V))


def sample_rows(logits: np.ndarray, uniforms, *, do_sample: bool = True, temperature: float = 1.0,
                top_p: float = 1.0, top_k: int | None = None) -> np.ndarray:
    x = _cf(logits)
    if x.ndim == 1:
        x = x[None]
    u = _cf(np.broadcast_to(np.asarray(uniforms, dtype=np.float32), (x.shape[0],)))
    out = np.zeros(x.shape[0], dtype=np.int32)
    lib().fgo_sample_rows(_p(x, _f32p), x.shape[1], x.shape[1], x.shape[0], _p(u, _f32p), int(bool(do_sample)),
                          float(temperature), float(top_p), int(top_k or 0), _p(out, _i32p))
    return out


def nucleus_kept(row: np.ndarray, temperature: float, top_p: float) -> np.ndarray:
    """fg-icdf-v1n kept set of one logits row (bool mask)."""
    r = _cf(row)
    mask = np.zeros(r.shape[0], dtype=np.uint8)
    lib().fgo_nucleus_kept(_p(r, _f32p), r.shape[0], float(temperature), float(top_p),
                           mask.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)))
    return mask.astype(bool)


def kept_set(row: np.ndarray, temperature: float, top_p: float, top_k: int | None) -> np.ndarray:
    """fg-icdf-v1n / v1k kept set of one logits row (bool mask)."""
    r = _cf(row)
    mask = np.zeros(r.shape[0], dtype=np.uint8)
    lib().fgo_kept_set(_p(r, _f32p), r.shape[0], float(temperature), float(top_p), int(top_k or 0),
                       mask.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)))
    return mask.astype(bool)


def topk_stable(row: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    r = _cf(row)
    idx = np.zeros(k, dtype=np.int32)
    val = np.zeros(k, dtype=np.float32)
    lib().fgo_topk_stable(_p(r, _f32p), r.shape[0], k, _p(idx, _i32p), _p(val, _f32p))
    return idx, val


def build_dense_trees(root, cand_idx: np.ndarray, topk_by_depth, budget: int, nmax: int) -> dict:
    root = _c32(root)
    B = root.shape[0]
    cand = _c32(cand_idx)  # [n_depth, B, kmax]
    n_depth = len(topk_by_depth)
    kmax = cand.shape[2] if cand.ndim == 3 else 1
    if n_depth == 0:
        cand = np.zeros((1, B, 1), dtype=np.int32)
        kmax = 1
    topk = _c32(list(topk_by_depth) or [0])
    tokens = np.zeros((B, nmax), dtype=np.int32)
    parents = np.zeros((B, nmax), dtype=np.int32)
    depths = np.zeros((B, nmax), dtype=np.int32)
    n_nodes = np.zeros(B, dtype=np.int32)
    lib().fgo_build_dense_trees(_p(root, _i32p), _p(cand, _i32p), kmax, _p(topk, _i32p), n_depth, budget, B, nmax,
                                _p(tokens, _i32p), _p(parents, _i32p), _p(depths, _i32p), _p(n_nodes, _i32p))
    return {"tokens": tokens, "parents": parents, "depths": depths, "n_nodes": n_nodes}


def accept_walk(logits: np.ndarray, slot, tokens, parents, n_nodes, uniforms, *, do_sample: bool, temperature: float,
                eos_id: int, max_length: int, row_len, dcap: int, top_p: float = 1.0,
                top_k: int | None = None) -> dict:
    x = _cf(logits)
    slot = _c32(slot)
    tokens = _c32(tokens)
    parents = _c32(parents)
    n_nodes = _c32(n_nodes)
    u = _cf(uniforms)
    row_len = _c32(row_len)
    B, nmax = tokens.shape
    out = {k: np.zeros((B, dcap), dtype=np.int32) for k in ("acc_tokens", "acc_nodes")}
    for k in ("acc_len", "raw_len", "correction", "pending", "last_node", "finished"):
        out[k] = np.zeros(B, dtype=np.int32)
    rc = lib().fgo_accept_walk(
        _p(x, _f32p), x.shape[1], x.shape[1], _p(slot, _i32p), _p(tokens, _i32p), _p(parents, _i32p),
        _p(n_nodes, _i32p), nmax, _p(u, _f32p), u.shape[1], B, int(bool(do_sample)), float(temperature),
        float(top_p), int(top_k or 0), eos_id,
        max_length, _p(row_len, _i32p), dcap, _p(out["acc_tokens"], _i32p), _p(out["acc_nodes"], _i32p),
        _p(out["acc_len"], _i32p), _p(out["raw_len"], _i32p), _p(out["correction"], _i32p),
        _p(out["pending"], _i32p), _p(out["last_node"], _i32p), _p(out["finished"], _i32p),
    )
    if rc != 0:
        raise ValueError(f"oracle walk: row {-rc - 1} visited a parent without a logits slot")
    return out


def extract_path(k_layers: list[np.ndarray], v_layers: list[np.ndarray], row_len, acc_nodes, acc_len) -> None:
    """In-place compaction on numpy caches shaped [B, Hkv, cap, D] (C-contiguous)."""
    row_len = _c32(row_len)
    acc_nodes = _c32(acc_nodes)
    acc_len = _c32(acc_len)
    ref = k_layers[0]
    B, H, cap, D = ref.shape
    for a in list(k_layers) + list(v_layers):
        assert a.flags["C_CONTIGUOUS"] and a.shape == ref.shape and a.dtype == ref.dtype
    kp = (ctypes.c_void_p * len(k_layers))(*[a.ctypes.data for a in k_layers])
    vp = (ctypes.c_void_p * len(v_layers))(*[a.ctypes.data for a in v_layers])
    lib().fgo_extract_path(kp, vp, len(k_layers), B, H, D, H * cap * D, cap * D, D, ref.dtype.itemsize,
                           _p(row_len, _i32p), _p(acc_nodes, _i32p), _p(acc_len, _i32p), acc_nodes.shape[1])

"""fg_tree_attention_noalloc against fg_tree_attention, through the C ABI.

The allocation-free entry point serves callers that cannot hand the library
device scratch memory (a runtime binding the C ABI without a device
allocator, or a memory manager that owns the GPU, where cudaMalloc would fail
or stall the device mid-round).  It must give the same attention output as
the regular entry point given caller-allocated scratch, on consecutive calls
that reuse its one built-in buffer.  This file is collected last so that a
run that stops at the first failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]


def _tree_anc(n: int, g: torch.Generator) -> torch.Tensor:
    parents = [-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, n)]
    bits = [[0, 0, 0, 0] for _ in range(n)]
    for i in range(n):
        j = i
        while j >= 0:
            bits[i][j >> 5] |= 1 << (j & 31)
            j = parents[j]
    t = torch.tensor(bits, dtype=torch.int64) & 0xFFFFFFFF
    return t.to(torch.uint32).view(torch.int32) if hasattr(torch, "uint32") else t.to(torch.int32)


def _call(lib, name, *args):
    from flashgrpo_b200 import _native

    status = getattr(lib, name)(*args)
    assert status == _native.FG_OK, (name, lib.fg_status_string(status).decode())


@pytest.mark.parametrize("B,n,hq,hkv,L,splits", [(8, 13, 12, 2, 1024, 3), (4, 32, 28, 4, 600, 0), (2, 64, 32, 8, 300, 2),
                                                  # the 256-row form (224 rows per KV head, 160 items); its
                                                  # split-K partials would outgrow the shared buffer
                                                  (40, 32, 28, 4, 300, 0)])
def test_noalloc_attention_matches_workspace_entry_point(B, n, hq, hkv, L, splits):
    from flashgrpo_b200 import _native, ops

    lib = _native.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator().manual_seed(B * 7 + n)
    D = 128
    cap = L + n + 8
    kv_len = torch.randint(max(L - 40, 0), L + 1, (B,), generator=g, dtype=torch.int32).to(dev)
    k = torch.randn(B, hkv, cap, D, generator=g).to(torch.bfloat16).to(dev)
    v = torch.randn(B, hkv, cap, D, generator=g).to(torch.bfloat16).to(dev)
    q = torch.randn(B, n, hq, D, generator=g).to(torch.bfloat16).to(dev)
    anc = _tree_anc(n, g).contiguous().to(dev)
    kv = ops.kv_layer(k, v)
    stream = torch.cuda.current_stream(dev).cuda_stream
    scale = D ** -0.5
    # regular entry point with scratch allocated by the caller
    need = int(lib.fg_tree_attention_workspace_size(B, n, hq, hkv, D, splits, L))
    ws = torch.zeros(max(need, 16) // 4 + 4, dtype=torch.int32, device=dev)
    ref = torch.empty_like(q)
    _call(lib, "fg_tree_attention", q.data_ptr(), _native.FG_DTYPE_BF16, ctypes.byref(kv), kv_len.data_ptr(),
          anc.data_ptr(), B, n, hq, hkv, D, scale, ref.data_ptr(), ws.data_ptr(), ws.numel() * 4, splits, L, stream)
    # allocation-free entry point, twice in a row on its shared buffer
    outs = []
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        _call(lib, "fg_tree_attention_noalloc", q.data_ptr(), _native.FG_DTYPE_BF16, ctypes.byref(kv),
              kv_len.data_ptr(), anc.data_ptr(), B, n, hq, hkv, D, scale, out.data_ptr(), splits, L, stream)
        outs.append(out)
    torch.cuda.synchronize(dev)
    # the same kernel with the same splits and a fixed merge order: bit for bit
    for out in outs:
        assert torch.isfinite(out.float()).all()
        assert torch.equal(out, ref)
    assert _native.read_device_error(clear=True) == 0


def test_noalloc_attention_fp32_needs_no_scratch():
    """fp32 calls use no scratch, so shapes whose bf16 split-K scratch would
    exceed the built-in array still run, and equal the regular entry point."""
    from flashgrpo_b200 import _native, ops

    lib = _native.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(5)
    B, n, hq, hkv, D, L = 3, 9, 8, 2, 64, 200
    cap = L + n + 4
    kv_len = torch.tensor([L, L - 17, 0], dtype=torch.int32, device=dev)
    k = torch.randn(B, hkv, cap, D, generator=g).to(dev)
    v = torch.randn(B, hkv, cap, D, generator=g).to(dev)
    q = torch.randn(B, n, hq, D, generator=g).to(dev)
    anc = _tree_anc(n, g).contiguous().to(dev)
    kv = ops.kv_layer(k, v)
    stream = torch.cuda.current_stream(dev).cuda_stream
    ref = torch.empty_like(q)
    _call(lib, "fg_tree_attention", q.data_ptr(), _native.FG_DTYPE_F32, ctypes.byref(kv), kv_len.data_ptr(),
          anc.data_ptr(), B, n, hq, hkv, D, D ** -0.5, ref.data_ptr(), None, 0, 0, L, stream)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        _call(lib, "fg_tree_attention_noalloc", q.data_ptr(), _native.FG_DTYPE_F32, ctypes.byref(kv),
              kv_len.data_ptr(), anc.data_ptr(), B, n, hq, hkv, D, D ** -0.5, out.data_ptr(), 0, L, stream)
        torch.cuda.synchronize(dev)
        assert torch.equal(out, ref)
    assert _native.read_device_error(clear=True) == 0


def test_noalloc_rejects_oversized_scratch():
    from flashgrpo_b200 import _native, ops

    lib = _native.load()
    dev = torch.device("cuda", 0)
    B, n, hq, hkv, D, cap = 256, 128, 32, 8, 128, 64
    k = torch.zeros(B, hkv, cap, D, dtype=torch.bfloat16, device=dev)
    q = torch.zeros(B, n, hq, D, dtype=torch.bfloat16, device=dev)
    kv = ops.kv_layer(k, k)
    kv_len = torch.zeros(B, dtype=torch.int32, device=dev)
    anc = torch.zeros(n, 4, dtype=torch.int32, device=dev)
    need = int(lib.fg_tree_attention_workspace_size(B, n, hq, hkv, D, 4, cap))
    assert need > _native.FG_NOALLOC_SCRATCH_BYTES
    status = lib.fg_tree_attention_noalloc(q.data_ptr(), _native.FG_DTYPE_BF16, ctypes.byref(kv), kv_len.data_ptr(),
                                           anc.data_ptr(), B, n, hq, hkv, D, 1.0, q.data_ptr(), 4, cap,
                                           torch.cuda.current_stream(dev).cuda_stream)
    assert status == _native.FG_ECAPACITY

"""CPU checks of the C ABI: the library loads and exports every declared symbol.

No kernel is launched (this container has no GPU).
"""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import REPO


def _declared_functions() -> list[str]:
    text = (REPO / "include" / "fg_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fg_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_hot_path():
    names = _declared_functions()
    for must in ("fg_sample_rows", "fg_row_topk", "fg_build_tree", "fg_tree_attention", "fg_accept_extract",
                 "fg_extract_path", "fg_rope_kv_write", "fg_philox_uniforms"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from flashgrpo_b200 import _native

    lib = _native.load()
    missing = [n for n in _declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_native.SIGNATURES) == set(_declared_functions())


def test_host_only_entry_points():
    from flashgrpo_b200 import _native

    lib = _native.load()
    assert lib.fg_version().decode().startswith("fg_b200")
    assert lib.fg_status_string(_native.FG_ETIMEOUT).decode() == "device wait timed out"
    # argument validation happens before any CUDA call
    assert lib.fg_sample_rows(None, 1, 10, 10, 3, None, 1, 1, 1.0, 1.0, 0, None, None, None) == _native.FG_EINVAL
    assert lib.fg_row_topk(ctypes.c_void_p(16), 1, 100, 100, 2, 99, ctypes.c_void_p(16), ctypes.c_void_p(16),
                           ctypes.c_void_p(16), ctypes.c_void_p(16), None) == _native.FG_ECAPACITY
    assert lib.fg_tree_attention_workspace_size(64, 13, 12, 2, 128, 1, 1024) == 0
    assert lib.fg_tree_attention_workspace_size(64, 13, 12, 2, 128, 2, 1024) > 0
    # fused lm_head + top-k: shape limits are checked before any CUDA call
    p = ctypes.c_void_p(256)
    lmh = lambda dtype, M, H, k: lib.fg_lm_head_topk(p, dtype, H, M, H, p, H, 1000, 0, None, 0, 0, k, p, p, p, None,
                                                      p, 1 << 20, None)
    assert lmh(_native.FG_DTYPE_F32, 64, 128, 4) == _native.FG_EUNSUPPORTED
    assert lmh(_native.FG_DTYPE_BF16, 257, 128, 4) == _native.FG_ECAPACITY
    assert lmh(_native.FG_DTYPE_BF16, 64, 100, 4) == _native.FG_ECAPACITY
    assert lib.fg_lm_head_topk_workspace_size(192, 151936, 64, 4) > 0
    assert lib.fg_lm_head_topk_workspace_size(192, 151936, 192, 4) == 0
    # MEDUSA proposal: dtype, row and width limits, head pointers, workspace
    heads = (_native.MedusaHead * 2)(*[_native.MedusaHead(256, 256, 256, 256)] * 2)
    prop = lambda dtype, B, H, hs, n, ws_bytes: lib.fg_medusa_propose(
        p, dtype, B, H, hs, n, 1e-5, p, H, 1000, p, 1000, 4, p, p, p, None, p, ws_bytes, None)
    big = 1 << 30
    assert prop(_native.FG_DTYPE_F32, 64, 128, heads, 2, big) == _native.FG_EUNSUPPORTED
    assert prop(_native.FG_DTYPE_BF16, 86, 128, heads, 2, big) == _native.FG_ECAPACITY    # 3 x 86 rows > 256
    assert prop(_native.FG_DTYPE_BF16, 64, 100, heads, 2, big) == _native.FG_ECAPACITY    # H not a multiple of 64
    assert prop(_native.FG_DTYPE_BF16, 64, 128, None, 2, big) == _native.FG_EINVAL
    bad = (_native.MedusaHead * 2)(_native.MedusaHead(256, 256, 256, 256), _native.MedusaHead(256, None, 256, 256))
    assert prop(_native.FG_DTYPE_BF16, 64, 128, bad, 2, big) == _native.FG_EINVAL
    assert prop(_native.FG_DTYPE_BF16, 64, 128, heads, 2, 1024) == _native.FG_ECAPACITY   # workspace too small
    need = lib.fg_medusa_propose_workspace_size(64, 1536, 151936, 2, 4)
    assert need >= 2 * 2 * 64 * 1536 * 2 + lib.fg_lm_head_topk_workspace_size(192, 151936, 64, 4)
    assert lib.fg_medusa_propose_workspace_size(64, 1536, 151936, 0, 4) == 256
    # chain step: dtype, widths, row grouping, overlap and workspace are checked before any CUDA call
    cell = _native.ChainCell(*([256] * 9), 192)
    step = lambda dtype, H, c, n_par, fan, n_ch, out, ws_bytes: lib.fg_chain_step(
        p, p, n_ch, 4, n_par, fan, n_ch, p, 2048, H, dtype, ctypes.byref(c), 1e-5, out, p, H, 1000, 4, p, p, p, None,
        p, ws_bytes, None)
    far = ctypes.c_void_p(1 << 40)
    assert step(_native.FG_DTYPE_F32, 1536, cell, 1, 4, 4, far, big) == _native.FG_EUNSUPPORTED
    assert step(_native.FG_DTYPE_BF16, 1536, cell, 1, 4, 5, far, big) == _native.FG_EINVAL      # 5 children > 1 x 4
    assert step(_native.FG_DTYPE_BF16, 1500, cell, 1, 4, 4, far, big) == _native.FG_ECAPACITY   # H % 64
    odd = _native.ChainCell(*([256] * 9), 100)
    assert step(_native.FG_DTYPE_BF16, 1536, odd, 1, 4, 4, far, big) == _native.FG_ECAPACITY    # bottleneck % 64
    assert step(_native.FG_DTYPE_BF16, 1536, cell, 1, 4, 4, p, big) == _native.FG_EINVAL        # state_out overlaps state
    assert step(_native.FG_DTYPE_BF16, 1536, cell, 1, 4, 4, far, 1024) == _native.FG_ECAPACITY  # workspace too small
    assert lib.fg_chain_step_workspace_size(512, 1536, 192, 151936, 4) == \
        lib.fg_chain_step_workspace_size(256, 1536, 192, 151936, 4)                           # 256-row passes
    # dense projections: dtype, K, N, tile and epilogue checks before any CUDA call
    lin = lambda dtype, M, K, N, bias, resid, ld, epi, bn, sp: lib.fg_linear(
        p, dtype, M, K, p, N, bias, resid, ld, p, ld, epi, 128, bn, sp, 0, None, 0, None)
    assert lin(_native.FG_DTYPE_F32, 64, 128, 64, None, None, 64, 0, 0, 0) == _native.FG_EUNSUPPORTED
    assert lin(_native.FG_DTYPE_BF16, 64, 100, 64, None, None, 64, 0, 0, 0) == _native.FG_ECAPACITY  # K % 64
    assert lin(_native.FG_DTYPE_BF16, 64, 128, 60, None, None, 60, 0, 0, 0) == _native.FG_EINVAL     # N % 8
    assert lin(_native.FG_DTYPE_BF16, 64, 128, 64, None, None, 64, 1, 0, 0) == _native.FG_EINVAL     # RESID needs resid
    assert lin(_native.FG_DTYPE_BF16, 64, 128, 64, p, None, 64, 2, 0, 0) == _native.FG_EINVAL        # no bias with SwiGLU
    assert lin(_native.FG_DTYPE_BF16, 64, 128, 64, None, None, 64, 0, 24, 1) == _native.FG_EINVAL    # bn % 16
    assert lin(_native.FG_DTYPE_BF16, 64, 128, 64, None, None, 64, 0, 16, 2) == _native.FG_ECAPACITY # split-K, no workspace
    assert lin(_native.FG_DTYPE_BF16, 64, 128, 64, None, None, 64, 7, 0, 0) == _native.FG_EINVAL     # epilogue
    assert lib.fg_linear(p, _native.FG_DTYPE_BF16, 64, 128, p, 64, None, None, 64, p, 64, 0, 192, 64, 1, 0, None, 0,
                         None) == _native.FG_EINVAL                                              # bm 128 or 256
    assert lib.fg_linear(p, _native.FG_DTYPE_BF16, 64, 128, p, 64, None, None, 64, p, 64, 0, 128, 64, 1, 9, None, 0,
                         None) == _native.FG_EINVAL                                              # ring stages
    assert lib.fg_linear_workspace_size(832, 1536, 8960, 1, 128, 256, 5) == 5 * 832 * 1536 * 4
    assert lib.fg_linear_workspace_size(832, 1536, 8960, 2, 256, 128, 3) == 3 * 832 * 2 * 1536 * 4
    assert lib.fg_linear_workspace_size(832, 1536, 8960, 1, 128, 256, 1) == 0


def test_plan_params_tables():
    from flashgrpo_b200 import ops

    p = ops.plan_params(tree_mode="concurrency_aware", active_batch_size=64, num_medusa_heads=3, cpeak_nodes=1024,
                        min_tree_nodes_per_seq=1, max_tree_nodes_per_seq=16, max_tree_depth=4,
                        fixed_tree_topk_by_depth=(4, 3, 2), adaptive_depth_weight_decay=0.5)
    assert p.tree_mode == 1 and p.n_fixed == 3 and list(p.fixed_topk)[:3] == [4, 3, 2]
    assert p.depth_weight[2] == 0.25
    import math

    assert p.log_gain[3] == math.log1p(3) - math.log(3)
    with pytest.raises(ValueError):
        ops.plan_params(tree_mode="sparse", active_batch_size=1, num_medusa_heads=1, cpeak_nodes=1,
                        min_tree_nodes_per_seq=1, max_tree_nodes_per_seq=1, max_tree_depth=2,
                        fixed_tree_topk_by_depth=(1,))


def test_ctypes_structures_match_the_header(tmp_path):
    """The ctypes mirrors of fg_plan_params, fg_kv_layer, fg_accept_args,
    fg_medusa_head and fg_chain_cell have the C structs' size and field offsets (compiled with gcc from the
    header)."""
    import shutil
    import subprocess

    from flashgrpo_b200 import _native as N

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = {"fg_plan_params": N.PlanParams, "fg_kv_layer": N.KvLayer, "fg_accept_args": N.AcceptArgs,
               "fg_medusa_head": N.MedusaHead, "fg_chain_cell": N.ChainCell}
    lines = []
    for cname, py in structs.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    src = tmp_path / "layout.c"
    src.write_text("#include <stddef.h>\n#include <stdio.h>\n#include \"fg_b200.h\"\nint main(void) {\n" +
                   "\n".join(lines) + "\nreturn 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(REPO / "include"), "-o", str(exe), str(src)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        cname, field, val = line.split()
        got[(cname, field)] = int(val)
    for cname, py in structs.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for f, _ in py._fields_:
            assert got[(cname, f)] == getattr(py, f).offset, (cname, f)

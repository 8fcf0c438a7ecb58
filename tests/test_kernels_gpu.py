"""GPU parity of every hot-path kernel, called through the C ABI.

Bit-exact against the CPU oracle: uniforms, sampling, top-k, tree build,
acceptance walk and KV compaction.  Within stated tolerances against a plain
PyTorch fp32 reference of the same op: tree attention, RoPE + KV write and
the elementwise layer pieces.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import cuda_available
from oracle import native as orc
from oracle import reference_path as rp

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]

DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    from flashgrpo_b200 import _native, ops as o

    _native.load()
    yield o
    assert _native.read_device_error(clear=True) == 0


def _to_np(t):
    return t.detach().float().cpu().numpy()


# ------------------------------------------------------------------ sampler
def test_philox_uniforms_bit_exact(ops):
    seq = torch.arange(0, 3000, 7, dtype=torch.int32, device=DEV)
    u = ops.philox_uniforms(0xDEADBEEF12345, seq, 17, 5)
    ref = orc.philox_uniforms(0xDEADBEEF12345, seq.cpu().numpy(), 17, 5)
    assert np.array_equal(u.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("V,temp,scale", [(4096, 1.0, 8.0), (151936, 1.0, 2.0), (97, 0.7, 3.0), (128256, 1.3, 1.0)])
def test_sample_rows_bit_exact(ops, dtype, V, temp, scale):
    g = torch.Generator().manual_seed(V + int(temp * 10))
    n = 24
    logits = (torch.randn(n, V, generator=g) * scale).to(dtype)
    u = torch.rand(n, generator=g)
    u[0], u[1] = 0.0, 1.0 - 2 ** -24
    got = ops.sample_rows(logits.to(DEV), u.to(DEV), temperature=temp).cpu().numpy()
    ref = orc.sample_rows(logits.float().numpy(), u.numpy(), temperature=temp)
    assert np.array_equal(got, ref)
    greedy = ops.sample_rows(logits.to(DEV), u.to(DEV), do_sample=False).cpu().numpy()
    assert np.array_equal(greedy, logits.float().argmax(-1).numpy())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("V,temp,scale,top_p", [(4096, 1.0, 8.0, 0.9), (151936, 1.0, 2.0, 0.95), (97, 0.7, 3.0, 0.5),
                                                (128256, 1.3, 1.0, 0.99), (1000, 1.0, 0.05, 0.8)])
def test_sample_rows_nucleus_bit_exact(ops, dtype, V, temp, scale, top_p):
    # fg-icdf-v1n: radix-select boundary on the GPU vs an explicit sort on the
    # CPU; bf16 rows have many tied values, so boundaries cut tie groups
    g = torch.Generator().manual_seed(V + int(temp * 10) + int(top_p * 100))
    n = 16
    logits = (torch.randn(n, V, generator=g) * scale).to(dtype)
    logits[2] = logits[2].round()  # heavy ties
    u = torch.rand(n, generator=g)
    u[0], u[1] = 0.0, 1.0 - 2 ** -24
    got = ops.sample_rows(logits.to(DEV), u.to(DEV), temperature=temp, top_p=top_p).cpu().numpy()
    ref = orc.sample_rows(logits.float().numpy(), u.numpy(), temperature=temp, top_p=top_p)
    assert np.array_equal(got, ref)
    for r in range(4):  # every draw lies in the kept set
        assert orc.nucleus_kept(logits[r].float().numpy(), temp, top_p)[got[r]]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("V,temp,scale,top_k,top_p", [(4096, 1.0, 8.0, 20, 1.0), (151936, 1.0, 2.0, 50, 1.0),
                                                      (151936, 0.8, 2.0, 40, 0.9), (97, 0.7, 3.0, 96, 0.5),
                                                      (1000, 1.0, 0.05, 1, 1.0), (128256, 1.3, 1.0, 300, 0.95)])
def test_sample_rows_topk_bit_exact(ops, dtype, V, temp, scale, top_k, top_p):
    # fg-icdf-v1k: the K-set by a count radix select on the GPU vs an explicit
    # sort on the CPU; the tied row puts the K-set boundary inside a tie group
    g = torch.Generator().manual_seed(V + top_k + int(top_p * 100))
    n = 16
    logits = (torch.randn(n, V, generator=g) * scale).to(dtype)
    logits[2] = logits[2].round()  # heavy ties
    u = torch.rand(n, generator=g)
    u[0], u[1] = 0.0, 1.0 - 2 ** -24
    got = ops.sample_rows(logits.to(DEV), u.to(DEV), temperature=temp, top_p=top_p, top_k=top_k).cpu().numpy()
    ref = orc.sample_rows(logits.float().numpy(), u.numpy(), temperature=temp, top_p=top_p, top_k=top_k)
    assert np.array_equal(got, ref)
    for r in range(4):
        assert orc.kept_set(logits[r].float().numpy(), temp, top_p, top_k)[got[r]]
    # top_k >= V is no cut: the fg-icdf-v1 / v1n draw
    same = ops.sample_rows(logits.to(DEV), u.to(DEV), temperature=temp, top_p=top_p, top_k=V).cpu().numpy()
    assert np.array_equal(same, orc.sample_rows(logits.float().numpy(), u.numpy(), temperature=temp, top_p=top_p))


def test_sample_rows_forced_and_strided(ops):
    logits = torch.randn(6, 3, 512).to(DEV)
    view = logits[:, 1, :]  # row stride 1536
    u = torch.rand(6, 4, device=DEV)
    forced = torch.tensor([-1, 7, -1, -1, 3, -1], dtype=torch.int32, device=DEV)
    got = ops.sample_rows(view, u, forced=forced).cpu().numpy()
    ref = orc.sample_rows(_to_np(view), _to_np(u[:, 0]))
    ref[1], ref[4] = 7, 3
    assert np.array_equal(got, ref)


def test_sampler_distribution_on_gpu(ops):
    n = 60_000
    logits = torch.log(torch.tensor([0.6, 0.4])).expand(n, 2).contiguous().to(DEV)
    u = ops.philox_uniforms(456, torch.arange(n, dtype=torch.int32, device=DEV), 0, 1)
    s = ops.sample_rows(logits, u).cpu()
    freq = torch.bincount(s.long(), minlength=2).float() / n
    assert torch.max(torch.abs(freq - torch.tensor([0.6, 0.4]))) < 0.015


# ------------------------------------------------------------------- top-k
@pytest.mark.parametrize("dtype,V,k", [(torch.bfloat16, 151936, 8), (torch.float32, 4096, 4), (torch.bfloat16, 97, 16),
                                       (torch.float16, 128256, 3)])
def test_row_topk_stable_and_lse(ops, dtype, V, k):
    g = torch.Generator().manual_seed(V)
    x = (torch.randn(20, V, generator=g) * 2).to(dtype)
    x[3, :] = 0.5  # every entry tied
    idx, val, mx, lse = ops.row_topk(x.to(DEV), k)
    for r in range(x.shape[0]):
        ri, rv = orc.topk_stable(x[r].float().numpy(), k)
        assert np.array_equal(idx[r].cpu().numpy(), ri), r
        assert np.array_equal(val[r].cpu().numpy(), rv), r
    assert torch.equal(mx.cpu(), x.float().max(-1).values)
    # fp32 logsumexp rounded to the logits dtype (torch's own fp16 reduction
    # overflows to inf on a flat 128k row, which the kernel does not copy)
    ref_lse = torch.logsumexp(x.to(DEV).float(), dim=-1).to(dtype).float().cpu()
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert torch.allclose(lse.cpu(), ref_lse, rtol=tol, atol=tol)


@pytest.mark.parametrize("dtype,V,k,rows", [(torch.bfloat16, 151936, 4, 128), (torch.bfloat16, 151936, 8, 9),
                                            (torch.float32, 4096, 1, 20), (torch.bfloat16, 97, 16, 5),
                                            (torch.float16, 128256, 2, 7), (torch.bfloat16, 13, 3, 3)])
def test_row_topk_without_lse_spreads_rows_over_clusters(ops, dtype, V, k, rows):
    """Without the logsumexp a row runs on an 8-CTA cluster (one vocabulary
    slice per CTA, merged through distributed shared memory): indices,
    values and maxima equal the CPU stable top-k and the one-CTA kernel's."""
    g = torch.Generator().manual_seed(V + k)
    x = (torch.randn(rows, V, generator=g) * 2).to(dtype)
    x[rows // 2, :] = 0.5  # every entry tied
    if V > 64:
        x[0, V - 3:] = 40.0  # the best entries in the last slice
    xd = x.to(DEV)
    idx, val, mx, lse = ops.row_topk(xd, k, with_lse=False)
    assert lse is None
    idx1, val1, mx1, _ = ops.row_topk(xd, k)
    assert torch.equal(idx, idx1) and torch.equal(val, val1) and torch.equal(mx, mx1)
    for r in range(rows):
        ri, rv = orc.topk_stable(x[r].float().numpy(), k)
        assert np.array_equal(idx[r].cpu().numpy(), ri), r
        assert np.array_equal(val[r].cpu().numpy(), rv), r
    # a strided view (rows of a wider buffer)
    wide = torch.zeros(rows, V + 64, dtype=dtype, device=DEV)
    wide[:, :V] = xd
    idx2, val2, mx2, _ = ops.row_topk(wide[:, :V], k, with_lse=False)
    assert torch.equal(idx2, idx1) and torch.equal(val2, val1)


# ---------------------------------------------------- fused lm_head + top-k
@pytest.mark.parametrize("M,H,V,n_write,row0,k,lse", [
    (192, 1536, 151936, 64, 64, 4, False),   # config 2: 64 root rows + 2 heads x 64 rows
    (192, 1536, 151936, 64, 64, 4, True),
    (130, 256, 5000, 2, 2, 8, True),         # second M block with 2 rows
    (64, 512, 1000, 0, 0, 16, True),         # V not a multiple of 16
    (256, 128, 32000, 256, 0, 2, False),     # all rows write logits and get top-k
    (7, 64, 300, 7, 3, 1, False),
    (40, 192, 2064, 40, 40, 4, False),       # logits only
])
def test_lm_head_topk_matches_gemm_then_row_topk(ops, M, H, V, n_write, row0, k, lse):
    g = torch.Generator().manual_seed(M * 31 + V)
    x = (torch.randn(M, H, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    w = (torch.randn(V, H, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    x[min(1, M - 1)] = 0  # an all-tied row: every logit is 0
    ref = (x.float() @ w.float().t())
    n_top = M - row0
    ws = torch.empty(max(ops.lm_head_topk_workspace_bytes(M, V, row0, k), 16) // 4 + 4, dtype=torch.int32, device=DEV)
    mk = lambda: (torch.empty((n_top, k), dtype=torch.int32, device=DEV),
                  torch.empty((n_top, k), dtype=torch.float32, device=DEV),
                  torch.empty(n_top, dtype=torch.float32, device=DEV),
                  torch.empty(n_top, dtype=torch.float32, device=DEV) if lse else None)
    # pass 1: every row's logits written, so the fused top-k can be checked
    # against fg_row_topk on exactly the values the kernel produced
    full = torch.full((M, V), float("nan"), dtype=torch.bfloat16, device=DEV)
    out1 = mk() if n_top > 0 else None
    ops.lm_head_topk(x, w, n_logit_rows=M, logits=full, topk_row0=row0, k=k, topk_out=out1, workspace=ws)
    torch.cuda.synchronize()
    assert torch.isfinite(full.float()).all()
    err = (full.float() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, err
    if n_top > 0:
        want = ops.row_topk(full[row0:], k, with_lse=lse)
        assert torch.equal(out1[0], want[0])
        assert torch.equal(out1[1], want[1])
        assert torch.equal(out1[2], want[2])
        if lse:
            assert torch.allclose(out1[3], want[3], rtol=1e-2, atol=1e-2)
    # pass 2: only the first n_write rows written; same top-k, same rows
    part = torch.full((M, V), float("nan"), dtype=torch.bfloat16, device=DEV)
    out2 = mk() if n_top > 0 else None
    ops.lm_head_topk(x, w, n_logit_rows=n_write, logits=part, topk_row0=row0, k=k, topk_out=out2, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(part[:n_write], full[:n_write])
    assert torch.isnan(part[n_write:].float()).all()
    if n_top > 0:
        for a, b in zip(out1, out2):
            if a is not None:
                assert torch.equal(a, b)


@pytest.mark.parametrize("B,H,V,n_heads,k,lse", [
    (64, 1536, 151936, 2, 4, False),   # config 2 proposal: 64 rows, 2 active heads
    (8, 3584, 152064, 3, 8, True),     # config 3 width (fc GEMMs wider than the SM count in 16-column units)
    (5, 256, 5000, 1, 2, True),        # ragged row count
    (16, 512, 3000, 0, 4, False),      # no heads: root logits only
    (20, 256, 2064, 9, 4, False),      # more heads than one LayerNorm launch serves, 200 rows
])
def test_medusa_propose_matches_torch_heads_then_lm_head(ops, B, H, V, n_heads, k, lse):
    """fg_medusa_propose: the heads' projected rows against
    MedusaPredictionHead.project_hidden evaluated by torch in bf16, and the
    lm_head part bit-identical to fg_lm_head_topk on the rows it produced."""
    F = torch.nn.functional
    bf = torch.bfloat16
    g = torch.Generator().manual_seed(B * 7 + H + n_heads)
    M = (1 + n_heads) * B
    x = torch.full((M, H), float("nan"), dtype=bf, device=DEV)
    x[:B] = (torch.randn(B, H, generator=g) * 0.5).to(bf).to(DEV)
    mk = lambda *shape, s=1.0, o=0.0: (torch.randn(*shape, generator=g) * s + o).to(bf).to(DEV)
    heads = [dict(norm_w=mk(H, s=0.1, o=1.0), norm_b=mk(H, s=0.1), fc_w=mk(H, H, s=H ** -0.5), fc_b=mk(H, s=0.1))
             for _ in range(n_heads)]
    w = mk(V, H, s=0.05)
    n_top = n_heads * B
    out = lambda: (torch.empty((n_top, k), dtype=torch.int32, device=DEV),
                   torch.empty((n_top, k), dtype=torch.float32, device=DEV),
                   torch.empty(n_top, dtype=torch.float32, device=DEV),
                   torch.empty(n_top, dtype=torch.float32, device=DEV) if lse else None) if n_heads else None
    root = torch.full((B, V), float("nan"), dtype=bf, device=DEV)
    ws = torch.empty(ops.medusa_propose_workspace_bytes(B, H, V, n_heads, k) // 4 + 64, dtype=torch.int32,
                     device=DEV)
    got = out()
    ops.medusa_propose(x, B, heads, w, root_logits=root, k=k, topk_out=got, workspace=ws)
    torch.cuda.synchronize()
    h = x[:B]
    h32 = h.float()
    for i, hw in enumerate(heads):
        got_i = x[(i + 1) * B:(i + 2) * B].float()
        # fp32 reference on the same bf16 inputs: the bf16 kernel within
        # 1e-2 relative in norm and no element further than 2e-2 of the
        # largest magnitude (the 2e-2 bf16 bound)
        w32 = {n: t.float() for n, t in hw.items()}
        ref32 = h32 + F.silu(F.linear(F.layer_norm(h32, (H,), w32["norm_w"], w32["norm_b"], 1e-5), w32["fc_w"],
                                      w32["fc_b"]))
        d32 = got_i - ref32
        assert (d32.norm() / ref32.norm()).item() <= 1e-2, i
        assert d32.abs().max().item() <= 2e-2 * ref32.abs().max().item(), i
        # and torch's own bf16 evaluation of the head within the same bounds
        ref = h + F.silu(F.linear(F.layer_norm(h, (H,), hw["norm_w"], hw["norm_b"], 1e-5), hw["fc_w"], hw["fc_b"]))
        d = got_i - ref.float()
        assert (d.norm() / ref.float().norm()).item() <= 1e-2, i
        assert d.abs().max().item() <= 2e-2 * ref.float().abs().max().item(), i
    want_root = torch.full((B, V), float("nan"), dtype=bf, device=DEV)
    want = out()
    lws = torch.empty(max(ops.lm_head_topk_workspace_bytes(M, V, B, k), 16) // 4 + 4, dtype=torch.int32, device=DEV)
    ops.lm_head_topk(x, w, n_logit_rows=B, logits=want_root, topk_row0=B, k=k, topk_out=want, workspace=lws)
    torch.cuda.synchronize()
    assert torch.equal(root, want_root)
    if n_heads:
        for a, b in zip(got, want):
            if a is not None:
                assert torch.equal(a, b)
    err = (root.float() - x[:B].float() @ w.float().t()).abs().max().item()
    assert err <= 1e-2 * root.float().abs().max().item() + 1e-3


def _chain_case(n_seq, n_parent, fanout, n_child, H, V, seed):
    bf = torch.bfloat16
    g = torch.Generator().manual_seed(seed)
    bn = max(64, H // 8)
    mk = lambda *shape, s=1.0, o=0.0: (torch.randn(*shape, generator=g) * s + o).to(bf).to(DEV)
    state = mk(n_seq * n_parent, H, s=0.5)
    tokens = torch.randint(0, V, (n_seq, n_parent * fanout), generator=g, dtype=torch.int32).to(DEV)
    embed = mk(V, H, s=0.05)
    cell = {"state_norm.weight": mk(H, s=0.1, o=1.0), "state_norm.bias": mk(H, s=0.1),
            "token_norm.weight": mk(H, s=0.1, o=1.0), "token_norm.bias": mk(H, s=0.1),
            "state_proj.weight": mk(bn, H, s=H ** -0.5), "token_proj.weight": mk(bn, H, s=H ** -0.5),
            "out_proj.weight": mk(H, bn, s=bn ** -0.5), "out_proj.bias": mk(H, s=0.1),
            "gate": torch.tensor(-1.0, dtype=bf, device=DEV)}
    return state, tokens, embed, cell


def _chain_ref(state, tokens, embed, cell, n_parent, fanout, n_child, fp32=False):
    """ChainDraftCell.forward evaluated by torch on the gathered rows, in
    bf16 (the inputs' dtype) or in fp32 on the same bf16 inputs."""
    F = torch.nn.functional
    if fp32:
        state, embed = state.float(), embed.float()
        cell = {n: t.float() for n, t in cell.items()}
    H = state.shape[1]
    M = tokens.shape[0] * n_child
    r = torch.arange(M, device=DEV)
    b, j = r // n_child, r % n_child
    s = state[b * n_parent + j // fanout]
    e = embed[tokens[b, j].long()]
    c = cell
    mixed = (F.linear(F.layer_norm(s, (H,), c["state_norm.weight"], c["state_norm.bias"], 1e-5),
                      c["state_proj.weight"])
             + F.linear(F.layer_norm(e, (H,), c["token_norm.weight"], c["token_norm.bias"], 1e-5),
                        c["token_proj.weight"]))
    delta = F.linear(F.silu(mixed), c["out_proj.weight"], c["out_proj.bias"])
    return s, s + torch.sigmoid(c["gate"]) * delta


@pytest.mark.parametrize("n_seq,n_parent,fanout,n_child,H,V,k", [
    (64, 4, 2, 8, 1536, 151936, 2),   # config-2 width, 512 rows: two 256-row passes
    (8, 1, 1, 1, 4096, 128256, 4),    # the cell on the root token, Llama-8B width (bottleneck 512)
    (5, 3, 3, 7, 512, 3000, 0),       # ragged children per parent, no top-k
])
def test_chain_step_matches_torch_cell_then_lm_head(ops, n_seq, n_parent, fanout, n_child, H, V, k):
    """fg_chain_step: the new states against torch's bf16 ChainDraftCell on
    the same parents and tokens, and the top-k bit-identical to
    fg_lm_head_topk on the states the call produced."""
    state, tokens, embed, cell = _chain_case(n_seq, n_parent, fanout, n_child, H, V, seed=n_seq + H)
    M = n_seq * n_child
    bn = cell["state_proj.weight"].shape[0]
    out = torch.full((M, H), float("nan"), dtype=torch.bfloat16, device=DEV)
    mk = lambda: (torch.empty((M, k), dtype=torch.int32, device=DEV), torch.empty((M, k), device=DEV),
                  torch.empty(M, device=DEV), torch.empty(M, device=DEV)) if k else None
    got = mk()
    ws = torch.empty(ops.chain_step_workspace_bytes(M, H, bn, V, k) // 4 + 64, dtype=torch.int32, device=DEV)
    ops.chain_step(state, tokens, n_parent=n_parent, fanout=fanout, n_child=n_child, embed=embed, cell=cell,
                   lm_head=embed if k else None, k=k, state_out=out, topk_out=got, workspace=ws)
    torch.cuda.synchronize()
    s, ref = _chain_ref(state, tokens, embed, cell, n_parent, fanout, n_child)
    d = out.float() - ref.float()
    # bf16 on both sides with different GEMM summation orders: the states
    # within 1e-2 normwise (no element beyond 2e-2 of the largest), and the
    # cell's update (state_out - parent) within 5e-2 normwise of torch's
    assert (d.norm() / ref.float().norm()).item() <= 1e-2
    assert d.abs().max().item() <= 2e-2 * ref.float().abs().max().item()
    upd, ref_upd = out.float() - s.float(), ref.float() - s.float()
    assert ((upd - ref_upd).norm() / ref_upd.norm()).item() <= 5e-2
    # the fp32 reference on the same bf16 inputs, within the same bounds
    s32, ref32 = _chain_ref(state, tokens, embed, cell, n_parent, fanout, n_child, fp32=True)
    d32 = out.float() - ref32
    assert (d32.norm() / ref32.norm()).item() <= 1e-2
    assert d32.abs().max().item() <= 2e-2 * ref32.abs().max().item()
    assert (((out.float() - s32) - (ref32 - s32)).norm() / (ref32 - s32).norm()).item() <= 5e-2
    if k:
        want = mk()
        ws2 = torch.empty(max(ops.lm_head_topk_workspace_bytes(256, V, 0, k), 16) // 4 + 4, dtype=torch.int32,
                          device=DEV)
        for r0 in range(0, M, 256):
            r1 = min(M, r0 + 256)
            ops.lm_head_topk(out[r0:r1], embed, n_logit_rows=0, logits=None, topk_row0=0, k=k,
                             topk_out=tuple(t[r0:r1] for t in want), workspace=ws2)
        torch.cuda.synchronize()
        for a, b in zip(got[:3], want[:3]):
            assert torch.equal(a, b)
        assert torch.allclose(got[3], want[3])


def test_chain_step_out_of_range_token_is_reported(ops):
    """A token outside [0, V) records FG_EINVAL in the device error word and
    reads embedding row 0 instead of memory outside the table."""
    from flashgrpo_b200 import _native

    state, tokens, embed, cell = _chain_case(2, 1, 2, 2, 256, 1000, seed=3)
    bad = tokens.clone()
    bad[1, 0] = 1000
    zero = tokens.clone()
    zero[1, 0] = 0
    ws = torch.empty(ops.chain_step_workspace_bytes(4, 256, 64, 1000, 0) // 4 + 64, dtype=torch.int32, device=DEV)
    outs = []
    assert _native.read_device_error(clear=True) == 0
    for t in (bad, zero):
        out = torch.empty((4, 256), dtype=torch.bfloat16, device=DEV)
        ops.chain_step(state, t, n_parent=1, fanout=2, n_child=2, embed=embed, cell=cell, lm_head=None, k=0,
                       state_out=out, topk_out=None, workspace=ws)
        torch.cuda.synchronize()
        outs.append(out)
        assert _native.read_device_error(clear=True) == (_native.FG_EINVAL if t is bad else 0)
    assert torch.equal(outs[0], outs[1])


# -------------------------------------------------------------- tree build
def _check_tree(ops, *, tree_mode, B, cpeak, mx, depth, fixed, n_heads, V=300, adaptive=False, amin=(1, 1, 1),
                metric="top1_prob", seed=0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    kw = dict(tree_mode=tree_mode, active_batch_size=B, num_medusa_heads=n_heads, cpeak_nodes=cpeak,
              min_tree_nodes_per_seq=1, max_tree_nodes_per_seq=mx, max_tree_depth=depth,
              fixed_tree_topk_by_depth=list(fixed), adaptive_tree_enabled=adaptive,
              adaptive_min_topk_by_depth=list(amin))
    plan = rp.plan_tree(**kw)
    head_logits = [(torch.randn(B, V, generator=g) * 3).to(dtype) for _ in range(max(plan.active_heads, 1))]
    head_logits[0][0, :5] = 10.0  # a tie at the top of one row
    root = torch.randint(0, V, (B,), generator=g, dtype=torch.int32)
    row_len = torch.randint(5, 300, (B,), generator=g, dtype=torch.int32)
    kmax = max(plan.topk_by_depth + [1])
    n_h = plan.active_heads
    cand = [ops.row_topk(h.to(DEV), kmax) for h in head_logits[:n_h]] if n_h else []
    cand_idx = torch.stack([c[0] for c in cand]) if n_h else None
    cand_val = torch.stack([c[1] for c in cand]) if n_h else None
    hmax = torch.stack([c[2] for c in cand]) if n_h else None
    hlse = torch.stack([c[3] for c in cand]) if n_h else None
    params = ops.plan_params(adaptive_confidence_metric=metric, **kw)
    nmax = 128
    out = ops.build_tree(params, root.to(DEV), cand_idx, cand_val, hmax, hlse, nmax=nmax, logits_dtype=dtype,
                         row_len=row_len.to(DEV))
    torch.cuda.synchronize()
    # oracle: same plan, same (optionally adapted) branching, stable top-k trees
    oplan = plan
    if adaptive and n_h:
        conf = rp.confidences([h.float() if dtype == torch.float32 else h for h in head_logits[:n_h]], metric, 0.25)
        adapted = [rp.topk_from_confidence(c, k, d, adaptive=True, min_topk_by_depth=amin, low=0.15, high=0.45)
                   for d, (k, c) in enumerate(zip(plan.topk_by_depth, conf))]
        adapted = rp.fit_topk_to_budget(adapted, plan.node_budget_per_seq, min_topk_by_depth=list(amin)[: len(adapted)])
        oplan = rp.Plan(plan.node_budget_per_seq, len(adapted), adapted, rp.dense_node_count(adapted), plan.mode)
    trees = rp.build_dense_trees(root.tolist(), [h.float() for h in head_logits[:n_h]], oplan)
    pl = out["plan"].cpu().tolist()
    n = trees[0].node_count
    assert pl[0] == oplan.node_budget_per_seq
    assert pl[10] == n
    got_tok = out["tokens"].cpu().numpy()
    for b, t in enumerate(trees):
        assert got_tok[b, :n].tolist() == t.tokens, b
    assert out["parents"][:n].tolist() == trees[0].parents
    assert out["depths"][:n].tolist() == trees[0].depths
    pos = out["positions"].cpu().numpy()
    for b in range(B):
        assert pos[b, :n].tolist() == [int(row_len[b]) + d - 1 for d in trees[0].depths]
    _, mask, _, _ = rp.tree_attention_inputs(trees[:1], torch.ones(1, 1, dtype=torch.long), torch.tensor([1]),
                                             pad_token_id=0, dtype=torch.float32)
    allowed = (mask[0, 0, :, 1:] == 0).numpy()
    anc = out["anc"].cpu().numpy().view(np.uint32)
    for i in range(n):
        bits = [(int(anc[i, j >> 5]) >> (j & 31)) & 1 for j in range(n)]
        assert bits == allowed[i, :n].astype(int).tolist(), i
    _, _, slots = rp.internal_logit_layout(trees)
    assert np.array_equal(out["slot"].cpu().numpy()[:, :n], np.array(slots))
    assert pl[11] == sum(1 for i in range(n) if trees[0].children.get(i))


@pytest.mark.parametrize("case", [
    dict(tree_mode="concurrency_aware", B=64, cpeak=1024, mx=16, depth=4, fixed=(4, 3, 2), n_heads=3),
    dict(tree_mode="fixed", B=4, cpeak=0, mx=16, depth=4, fixed=(4, 2, 2), n_heads=3),
    dict(tree_mode="concurrency_aware", B=16, cpeak=512, mx=32, depth=5, fixed=(3, 3, 2, 1), n_heads=4),
    dict(tree_mode="concurrency_aware", B=2, cpeak=4096, mx=128, depth=6, fixed=(2, 2, 2, 2, 2), n_heads=5),
    dict(tree_mode="concurrency_aware", B=256, cpeak=512, mx=10, depth=4, fixed=(4, 3, 2), n_heads=3),
    dict(tree_mode="concurrency_aware", B=16, cpeak=512, mx=32, depth=4, fixed=(8, 8, 8), n_heads=3, adaptive=True,
         amin=(2, 2, 2)),
    dict(tree_mode="concurrency_aware", B=100, cpeak=3200, mx=32, depth=5, fixed=(8, 8, 8, 8), n_heads=4,
         adaptive=True, amin=(1, 1, 1, 1), metric="margin"),
    dict(tree_mode="concurrency_aware", B=8, cpeak=64, mx=16, depth=4, fixed=(4, 3, 2), n_heads=3,
         dtype=torch.float32),
])
def test_build_tree_matches_oracle(ops, case):
    _check_tree(ops, **case)


# ------------------------------------------------ acceptance + compaction
def _run_accept(ops, logits, slots, tokens, parents, n_nodes, uniforms, *, do_sample, temperature, row_len,
                max_length=1 << 30, eos=-7, dcap=8, k_layers=(), v_layers=(), tree_hidden=None, hidden_out=None,
                top_p=1.0, top_k=None, kv_rows=None, parallel=None):
    B = tokens.shape[0]
    outs = {k: torch.full((B, dcap), -9, dtype=torch.int32, device=DEV) for k in ("acc_tokens", "acc_nodes")}
    for k in ("acc_len", "correction", "pending", "last_node", "finished"):
        outs[k] = torch.full((B,), -9, dtype=torch.int32, device=DEV)
    rl = row_len.clone()
    acc_total = torch.full((1,), 5, dtype=torch.int64, device=DEV)
    round_counter = torch.full((1,), 11, dtype=torch.int32, device=DEV)
    ops.accept_extract(logits=logits, slot=slots, tokens=tokens, parents=parents, n_nodes=n_nodes,
                       uniforms=uniforms, do_sample=do_sample, temperature=temperature, eos_id=eos,
                       max_length=max_length, row_len=rl, outputs=outs, dcap=dcap, parents_shared=parallel is not None,
                       k_layers=k_layers, v_layers=v_layers, tree_hidden=tree_hidden, hidden_out=hidden_out,
                       top_p=top_p, top_k=top_k, kv_rows=kv_rows, parallel=parallel, acc_total=acc_total,
                       round_counter=round_counter)
    torch.cuda.synchronize()
    # the round counters: accepted tokens added up, one round counted
    assert int(acc_total) == 5 + int(outs["acc_len"].sum())
    assert int(round_counter) == 12
    return outs, rl


def test_accept_matches_reference_fixture(ops, golden_dir):
    g = np.load(golden_dir / "accept.npz")
    for c in sorted({k.split("_")[0] for k in g.files}):
        V, B, nmax, do_sample = g[c + "_meta"].tolist()
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
        outs, _ = _run_accept(ops, t(g[c + "_logits"]), t(g[c + "_slots"]), t(g[c + "_tokens"]),
                              t(g[c + "_parents"]), t(g[c + "_n_nodes"]), t(g[c + "_uniforms"]),
                              do_sample=bool(do_sample), temperature=float(g[c + "_temp"][0]),
                              row_len=torch.zeros(B, dtype=torch.int32, device=DEV), dcap=5)
        assert np.array_equal(outs["acc_tokens"].cpu().numpy(), g[c + "_acc_tokens"]), c
        assert np.array_equal(outs["acc_nodes"].cpu().numpy(), g[c + "_acc_nodes"]), c
        assert np.array_equal(outs["correction"].cpu().numpy(), g[c + "_correction"]), c
        assert np.array_equal(outs["last_node"].cpu().numpy(), g[c + "_parent"]), c


@pytest.mark.parametrize("parallel", [False, True])
@pytest.mark.parametrize("dtype,V,B,peak,top_p,top_k", [
    (torch.bfloat16, 151936, 64, 6.0, 1.0, None), (torch.float32, 4096, 12, 8.0, 1.0, None),
    (torch.float16, 1000, 33, 5.0, 1.0, None), (torch.bfloat16, 151936, 64, 6.0, 0.9, None),
    (torch.float32, 4096, 12, 2.0, 0.5, None),
    # rows of an odd length: the scalar paths of the clustered draw
    (torch.bfloat16, 1001, 9, 5.0, 1.0, None),
    # 8 rows x 5 parents x 8 = 320 chunk-group loads in flight
    (torch.bfloat16, 40000, 8, 3.0, 1.0, None),
    # top-k draws (fg-icdf-v1k), alone and with a top_p cut
    (torch.bfloat16, 151936, 64, 6.0, 1.0, 50), (torch.float32, 4096, 12, 2.0, 0.8, 20)])
def test_accept_extract_random_bit_exact(ops, dtype, V, B, peak, top_p, top_k, parallel):
    """K4 against the oracle walk, bit for bit: drawing during the walk, and
    (parallel) every internal node's draw made before the walk on the shared
    topology."""
    g = torch.Generator().manual_seed(V + B)
    plan = rp.Plan(16, 3, [4, 2, 2], 0, "fixed")
    heads = [(torch.randn(B, V, generator=g) * peak).to(dtype).float() for _ in range(3)]
    root = torch.randint(0, V, (B,), generator=g)
    trees = rp.build_dense_trees(root.tolist(), heads, plan)
    n = trees[0].node_count
    rows, nodes, slots = rp.internal_logit_layout(trees)
    packed = torch.stack([heads[min(trees[r].depths[nd] - 1, 2)][r] for r, nd in zip(rows, nodes)])
    packed = (packed + torch.randn(packed.shape, generator=g) * 0.3).to(dtype)
    tok = torch.tensor([t.tokens for t in trees], dtype=torch.int32)
    par = torch.tensor([t.parents for t in trees], dtype=torch.int32)
    U = torch.rand(B, 6, generator=g)
    row_len = torch.randint(40, 60, (B,), generator=g, dtype=torch.int32)
    max_length = 58
    eos = int(tok[0, 1])
    # caches: 3 layers, [B, 2, cap, 128]
    cap = 96
    kl = [torch.randn(B, 2, cap, 128, generator=g).to(torch.bfloat16).to(DEV) for _ in range(3)]
    vl = [torch.randn(B, 2, cap, 128, generator=g).to(torch.bfloat16).to(DEV) for _ in range(3)]
    k_np = [k.view(torch.int16).cpu().numpy().copy() for k in kl]
    v_np = [v.view(torch.int16).cpu().numpy().copy() for v in vl]
    hidden = torch.randn(B, n, 64, generator=g).to(DEV)
    hout = torch.zeros(B, 64, device=DEV)
    par_arg, par_in = par.to(DEV), None
    if parallel:
        # dense trees of one plan share their topology
        assert all(t.parents == trees[0].parents for t in trees)
        internal = [i for i in range(n) if trees[0].children.get(i)]
        par_arg = par[0].contiguous().to(DEV)
        par_in = (torch.tensor(internal, dtype=torch.int32, device=DEV),
                  torch.tensor(trees[0].depths, dtype=torch.int32, device=DEV), None,
                  torch.full((packed.shape[0],), -9, dtype=torch.int32, device=DEV))
    outs, rl = _run_accept(ops, packed.to(DEV), torch.tensor(slots, dtype=torch.int32).to(DEV), tok.to(DEV),
                           par_arg, torch.full((B,), n, dtype=torch.int32, device=DEV), U.to(DEV),
                           do_sample=True, temperature=1.0, row_len=row_len.to(DEV), max_length=max_length, eos=eos,
                           dcap=8, k_layers=kl, v_layers=vl, tree_hidden=hidden, hidden_out=hout, top_p=top_p,
                           top_k=top_k, parallel=par_in)
    ref = orc.accept_walk(packed.float().numpy(), np.array(slots), tok.numpy(), par.numpy(), np.full(B, n), U.numpy(),
                          do_sample=True, temperature=1.0, eos_id=eos, max_length=max_length,
                          row_len=row_len.numpy(), dcap=8, top_p=top_p, top_k=top_k)
    for k in ("acc_tokens", "acc_nodes", "acc_len", "correction", "pending", "last_node", "finished"):
        assert np.array_equal(outs[k].cpu().numpy(), ref[k]), k
    assert np.array_equal(rl.cpu().numpy(), row_len.numpy() + ref["acc_len"])
    orc.extract_path(k_np, v_np, row_len.numpy(), ref["acc_nodes"], ref["acc_len"])
    for li in range(3):
        assert np.array_equal(kl[li].view(torch.int16).cpu().numpy(), k_np[li]), li
        assert np.array_equal(vl[li].view(torch.int16).cpu().numpy(), v_np[li]), li
    want_h = hidden[torch.arange(B), torch.from_numpy(ref["last_node"]).long().to(DEV)]
    assert torch.equal(hout, want_h)


def test_extract_path_standalone_matches_reference_fixture(ops, golden_dir):
    g = np.load(golden_dir / "extract.npz")
    for c in sorted({k.split("_")[0] for k in g.files}):
        B, H, old, n, D, is_bf16 = g[c + "_meta"].tolist()
        paths = g[c + "_paths"]
        lens = (paths >= 0).sum(1).astype(np.int32)
        conv = (lambda a: torch.from_numpy(a).view(torch.bfloat16)) if is_bf16 else torch.from_numpy
        ks = [conv(g[c + f"_k{i}"].copy()).to(DEV) for i in range(2)]
        vs = [conv(g[c + f"_v{i}"].copy()).to(DEV) for i in range(2)]
        if (D * ks[0].element_size()) % 16:
            continue
        ops.extract_path(ks, vs, torch.full((B,), old, dtype=torch.int32, device=DEV),
                         torch.from_numpy(np.where(paths < 0, 0, paths).astype(np.int32)).to(DEV),
                         torch.from_numpy(lens).to(DEV))
        torch.cuda.synchronize()
        for i in range(2):
            rk = conv(g[c + f"_rk{i}"].copy())
            rv = conv(g[c + f"_rv{i}"].copy())
            for b in range(B):
                a = old + lens[b]
                assert torch.equal(ks[i][b, :, :a].cpu(), rk[b, :, :a]), (c, i, b)
                assert torch.equal(vs[i][b, :, :a].cpu(), rv[b, :, :a]), (c, i, b)


# ---------------------------------------------------------- tree attention
def _random_tree(n, g):
    parents = [-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, n)]
    return rp.Tree(list(range(n)), parents, [1] * n)


def _anc_bits(tree, n):
    bits = torch.zeros(n, 4, dtype=torch.int64)
    for i in range(n):
        for a in tree.ancestors_including_self(i):
            bits[i, a >> 5] |= 1 << (a & 31)
    return (bits & 0xFFFFFFFF).to(torch.int64).numpy().astype(np.uint32).view(np.int32)


def _attn_reference(q, k, v, kv_len, tree, scale):
    """fp32 eager attention with the reference's additive mask, per row."""
    B, n, hq, D = q.shape
    hkv = k.shape[1]
    G = hq // hkv
    out = torch.zeros(B, n, hq, D, dtype=torch.float32, device=q.device)
    allowed_tree = torch.zeros(n, n, dtype=torch.bool)
    for i in range(n):
        for a in tree.ancestors_including_self(i):
            allowed_tree[i, a] = True
    for b in range(B):
        L = int(kv_len[b])
        kk = k[b, :, : L + n].float().repeat_interleave(G, 0)  # [hq, T, D]
        vv = v[b, :, : L + n].float().repeat_interleave(G, 0)
        qq = q[b].float().transpose(0, 1)  # [hq, n, D]
        s = torch.matmul(qq, kk.transpose(1, 2)) * scale
        mask = torch.cat([torch.ones(n, L, dtype=torch.bool), allowed_tree], 1).to(q.device)
        s = s.masked_fill(~mask, torch.finfo(torch.float32).min)
        out[b] = torch.matmul(torch.softmax(s, -1), vv).transpose(0, 1)
    return out


@pytest.mark.parametrize("B,n,hq,hkv,L,splits", [
    (8, 13, 12, 2, 1024, 0), (8, 13, 12, 2, 1024, 1), (4, 13, 12, 2, 700, 3), (6, 32, 28, 4, 517, 0),
    (2, 64, 32, 8, 300, 2), (3, 128, 32, 8, 129, 0), (1, 16, 32, 8, 4000, 0), (5, 1, 12, 2, 63, 0),
    (2, 8, 8, 8, 0, 0), (64, 13, 12, 2, 1024, 0), (1, 16, 32, 8, 4000, 24), (2, 13, 12, 2, 1500, 64),
    # config-5 sweep corners: the longest prefix with the fewest nodes, a long
    # prefix with 4 query-row groups per KV head
    (1, 8, 32, 8, 32768, 0), (2, 128, 32, 8, 16384, 0),
    # 129-256 query rows per KV head on >= 148 (row, head) items: the wide
    # kernel (two 128-row halves per CTA, P in TMEM), whole and with 3 splits
    (19, 64, 32, 8, 300, 0), (19, 53, 32, 8, 1500, 3), (37, 32, 28, 4, 517, 0),
])
def test_tree_attention_bf16(ops, B, n, hq, hkv, L, splits):
    g = torch.Generator().manual_seed(B * 1000 + n)
    D = 128
    cap = L + n + 40
    kv_len = torch.randint(max(L - 60, 0), L + 1, (B,), generator=g, dtype=torch.int32)
    k = torch.randn(B, hkv, cap, D, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(B, hkv, cap, D, generator=g).to(torch.bfloat16).to(DEV)
    q = torch.randn(B, n, hq, D, generator=g).to(torch.bfloat16).to(DEV)
    tree = _random_tree(n, g)
    anc = torch.from_numpy(_anc_bits(tree, n)).to(DEV)
    ws_bytes = ops.attention_workspace_bytes(B, n, hq, hkv, D, num_splits=splits, max_kv_len=int(kv_len.max()))
    ws = torch.zeros(max(ws_bytes, 16) // 4 + 4, dtype=torch.int32, device=DEV)
    scale = D ** -0.5
    out = ops.tree_attention(q, k, v, kv_len.to(DEV), anc, scale=scale, workspace=ws, num_splits=splits,
                             max_kv_len=int(kv_len.max()))
    ref = _attn_reference(q, k, v, kv_len, tree, scale)
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * max(ref.abs().max().item(), 1e-3), err
    # a second call reuses the (self-resetting) workspace
    out2 = ops.tree_attention(q, k, v, kv_len.to(DEV), anc, scale=scale, workspace=ws, num_splits=splits,
                              max_kv_len=int(kv_len.max()))
    assert torch.equal(out, out2)


def test_tree_attention_f32(ops):
    g = torch.Generator().manual_seed(3)
    B, n, hq, hkv, D, L = 4, 13, 4, 2, 64, 128
    k = torch.randn(B, hkv, L + n, D, generator=g).to(DEV)
    v = torch.randn(B, hkv, L + n, D, generator=g).to(DEV)
    q = torch.randn(B, n, hq, D, generator=g).to(DEV)
    kv_len = torch.full((B,), L, dtype=torch.int32)
    tree = _random_tree(n, g)
    anc = torch.from_numpy(_anc_bits(tree, n)).to(DEV)
    out = ops.tree_attention(q, k, v, kv_len.to(DEV), anc, scale=D ** -0.5)
    ref = _attn_reference(q.double(), k.double(), v.double(), kv_len, tree, D ** -0.5)
    rel = ((out - ref).abs().max() / ref.abs().max()).item()
    assert rel < 1e-5, rel


# ------------------------------------------------------------ layer pieces
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rope_kv_write_matches_hf(ops, dtype):
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    g = torch.Generator().manual_seed(5)
    B, n, hq, hkv, D, cap = 3, 13, 12, 2, 128, 300
    qkv = torch.randn(B * n, (hq + 2 * hkv) * D, generator=g).to(dtype).to(DEV)
    kv_len = torch.tensor([100, 7, 250], dtype=torch.int32, device=DEV)
    positions = (kv_len[:, None] + torch.randint(0, 4, (1, n), generator=g).to(DEV)).to(torch.int32)
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    kc = torch.zeros(B, hkv, cap, D, dtype=dtype, device=DEV)
    vc = torch.zeros_like(kc)
    q_out = torch.empty(B, n, hq, D, dtype=dtype, device=DEV)
    ops.rope_kv_write(qkv, positions, inv_freq.to(DEV), 1.0, B=B, n_nodes=n, n_q_heads=hq, n_kv_heads=hkv,
                      head_dim=D, kv_len=kv_len, k_cache=kc, v_cache=vc, q_out=q_out)
    # the per-round cos/sin table path (vectorized kernel) gives the same bits
    table = ops.rope_table(positions, inv_freq.to(DEV), 1.0, dtype)
    kc2, vc2, q2 = torch.zeros_like(kc), torch.zeros_like(vc), torch.empty_like(q_out)
    ops.rope_kv_write(qkv, positions, inv_freq.to(DEV), 1.0, B=B, n_nodes=n, n_q_heads=hq, n_kv_heads=hkv,
                      head_dim=D, kv_len=kv_len, k_cache=kc2, v_cache=vc2, q_out=q2, cos_sin=table)
    assert torch.equal(q2, q_out) and torch.equal(kc2, kc) and torch.equal(vc2, vc)
    # HF reference: cos/sin in fp32 -> activation dtype, rotate in that dtype
    freqs = positions.float()[..., None] * inv_freq.to(DEV)
    emb = torch.cat([freqs, freqs], -1)
    cos, sin = emb.cos().to(dtype), emb.sin().to(dtype)  # [B, n, D]
    x = qkv.view(B, n, hq + 2 * hkv, D).transpose(1, 2)
    qr, kr = apply_rotary_pos_emb(x[:, :hq], x[:, hq:hq + hkv], cos, sin)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert torch.allclose(q_out.float(), qr.transpose(1, 2).float(), atol=tol, rtol=tol)
    for b in range(B):
        L = int(kv_len[b])
        assert torch.allclose(kc[b, :, L:L + n].float(), kr[b].float(), atol=tol, rtol=tol)
        assert torch.equal(vc[b, :, L:L + n], x[b, hq + hkv:])
        assert torch.count_nonzero(kc[b, :, :L]) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_row_map_matches_gathered_cache(ops, dtype):
    """Retired rows: RoPE/KV write, tree attention and the accept compaction
    over a subset of the cache's rows through the row map (fg_kv_layer.rows,
    kv_rows) give the bits of the same calls on a gathered copy of those rows
    and leave every other row untouched."""
    g = torch.Generator().manual_seed(21)
    Bc, n, hq, hkv, D, cap = 7, 13, 12, 2, 128, 320
    rows = [5, 0, 3, 6]
    others = [r for r in range(Bc) if r not in rows]
    B = len(rows)
    rows_d = torch.tensor(rows, dtype=torch.int32, device=DEV)
    kc = torch.randn(Bc, hkv, cap, D, generator=g).to(dtype).to(DEV)
    vc = torch.randn(Bc, hkv, cap, D, generator=g).to(dtype).to(DEV)
    kv_len = torch.randint(150, 290, (B,), generator=g, dtype=torch.int32).to(DEV)
    # --- RoPE + tree K/V write (scalar path, and the cos/sin table path for bf16)
    qkv = torch.randn(B * n, (hq + 2 * hkv) * D, generator=g).to(dtype).to(DEV)
    positions = (kv_len[:, None] + torch.arange(n, device=DEV)[None]).to(torch.int32)
    inv_freq = (1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))).to(DEV)
    tables = [None] + ([ops.rope_table(positions, inv_freq, 1.0, dtype)] if dtype == torch.bfloat16 else [])
    for table in tables:
        kg, vg = kc[rows].clone(), vc[rows].clone()
        km, vm = kc.clone(), vc.clone()
        q1, q2 = (torch.empty(B, n, hq, D, dtype=dtype, device=DEV) for _ in range(2))
        common = dict(B=B, n_nodes=n, n_q_heads=hq, n_kv_heads=hkv, head_dim=D, kv_len=kv_len, cos_sin=table)
        ops.rope_kv_write(qkv, positions, inv_freq, 1.0, k_cache=kg, v_cache=vg, q_out=q1, **common)
        ops.rope_kv_write(qkv, positions, inv_freq, 1.0, k_cache=None, v_cache=None, q_out=q2,
                          kv=ops.kv_layer(km, vm, rows=rows_d), **common)
        torch.cuda.synchronize()
        assert torch.equal(q1, q2)
        assert torch.equal(km[rows], kg) and torch.equal(vm[rows], vg)
        assert torch.equal(km[others], kc[others]) and torch.equal(vm[others], vc[others])
    kc, vc = km, vm
    # --- tree attention over the mapped rows (one and several splits for bf16)
    tree = _random_tree(n, g)
    anc = torch.from_numpy(_anc_bits(tree, n)).to(DEV)
    q = torch.randn(B, n, hq, D, generator=g).to(dtype).to(DEV)
    kg, vg = kc[rows].contiguous(), vc[rows].contiguous()
    for splits in ([0, 3] if dtype == torch.bfloat16 else [0]):
        ws_bytes = ops.attention_workspace_bytes(B, n, hq, hkv, D, num_splits=splits, max_kv_len=cap)
        ws = torch.zeros(max(ws_bytes, 16) // 4 + 4, dtype=torch.int32, device=DEV)
        o1 = ops.tree_attention(q, kg, vg, kv_len, anc, scale=D ** -0.5, workspace=ws, num_splits=splits,
                                max_kv_len=cap)
        o2 = ops.tree_attention(q, kc, vc, kv_len, anc, scale=D ** -0.5, workspace=ws, num_splits=splits,
                                max_kv_len=cap, kv=ops.kv_layer(kc, vc, rows=rows_d))
        torch.cuda.synchronize()
        assert torch.equal(o1, o2), splits
    if dtype != torch.bfloat16:
        return
    # --- acceptance + extract_path compaction of the mapped rows
    V = 512
    plan = rp.Plan(16, 3, [4, 2, 2], 0, "fixed")
    # one peaked distribution for every depth: the draws usually match a child
    h = (torch.randn(B, V, generator=g) * 8).to(dtype).float()
    heads = [h, h, h]
    root = torch.randint(0, V, (B,), generator=g)
    trees = rp.build_dense_trees(root.tolist(), heads, plan)
    nn = trees[0].node_count
    trows, tnodes, slots = rp.internal_logit_layout(trees)
    packed = torch.stack([heads[min(trees[r].depths[nd] - 1, 2)][r] for r, nd in zip(trows, tnodes)]).to(dtype)
    tok = torch.tensor([t.tokens for t in trees], dtype=torch.int32).to(DEV)
    par = torch.tensor([t.parents for t in trees], dtype=torch.int32).to(DEV)
    U = torch.rand(B, 6, generator=g).to(DEV)
    layers_g = [(kc[rows].clone(), vc[rows].clone()) for _ in range(2)]
    layers_m = [(kc.clone(), vc.clone()) for _ in range(2)]
    args = (ops, packed.to(DEV), torch.tensor(slots, dtype=torch.int32).to(DEV), tok, par,
            torch.full((B,), nn, dtype=torch.int32, device=DEV), U)
    o_g, rl_g = _run_accept(*args, do_sample=True, temperature=1.0, row_len=kv_len, k_layers=[k for k, _ in layers_g],
                            v_layers=[v for _, v in layers_g])
    o_m, rl_m = _run_accept(*args, do_sample=True, temperature=1.0, row_len=kv_len, k_layers=[k for k, _ in layers_m],
                            v_layers=[v for _, v in layers_m], kv_rows=rows_d)
    for key in o_g:
        assert torch.equal(o_g[key], o_m[key]), key
    assert torch.equal(rl_g, rl_m)
    assert int(o_g["acc_len"].max()) >= 2  # some row moved slots
    for (kg_, vg_), (km_, vm_) in zip(layers_g, layers_m):
        assert torch.equal(km_[rows], kg_) and torch.equal(vm_[rows], vg_)
        assert torch.equal(km_[others], kc[others]) and torch.equal(vm_[others], vc[others])


@pytest.mark.parametrize("T,H,I", [
    (832, 1536, 8960),   # config 2: 64 rows x 13 tree nodes, Qwen2.5-1.5B MLP
    (100, 256, 384),     # one partial token tile
    (300, 512, 1024),    # three token tiles, the last partial
])
def test_gate_up_silu_matches_gemm_then_silu_mul(ops, T, H, I):
    """fg_gate_up_silu against torch's bf16 gate/up GEMM followed by
    fg_silu_mul on the materialized [T, 2I] tensor (both round g and u to
    bf16 before the gating; only the GEMM summation order differs)."""
    g = torch.Generator().manual_seed(T + I)
    x = (torch.randn(T, H, generator=g)).to(torch.bfloat16).to(DEV)
    w = (torch.randn(2 * I, H, generator=g) * H ** -0.5).to(torch.bfloat16).to(DEV)
    out = torch.full((T, I), float("nan"), dtype=torch.bfloat16, device=DEV)
    got = ops.gate_up_silu(x, w, out=out)
    ref = ops.silu_mul(x @ w.t())
    torch.cuda.synchronize()
    assert torch.isfinite(got.float()).all()
    d = got.float() - ref.float()
    assert (d.norm() / ref.float().norm()).item() <= 1e-2
    assert d.abs().max().item() <= 2e-2 * ref.float().abs().max().item()
    # a second call into the same buffer gives the same bits
    again = ops.gate_up_silu(x, w, out=torch.empty_like(out))
    torch.cuda.synchronize()
    assert torch.equal(again, got)


def _linear_ref(x, w, epi, bias=None, resid=None):
    """fp32 reference of fg_linear's epilogues (SwiGLU rounds g and u to bf16
    as the HF MLP's bf16 linears do before act_fn)."""
    d = x.float() @ w.float().t()
    if epi == 2:
        n = w.shape[0] // 2
        gb, ub = d[:, :n].bfloat16().float(), d[:, n:].bfloat16().float()
        return torch.nn.functional.silu(gb) * ub
    if bias is not None:
        d = d + bias.float()
    if resid is not None:
        d = d + resid.float()
    return d


@pytest.mark.parametrize("M,K,N,epi,bias,bm,bn,splits", [
    (832, 1536, 2048, 0, True, 0, 0, 0),         # config 2 QKV with bias
    (832, 1536, 1536, 1, False, 0, 0, 0),        # O projection + residual, in place
    (832, 8960, 1536, 1, False, 0, 0, 0),        # down projection + residual
    (832, 1536, 8960, 2, False, 0, 0, 0),        # gate/up + SwiGLU
    (320, 1536, 151936, 0, False, 0, 0, 0),      # internal-node lm_head (5 x 64 rows)
    (77, 256, 200, 1, True, 128, 48, 2),         # partial token and output tiles, split-K
    (300, 512, 1024, 2, False, 128, 64, 4),      # SwiGLU with split-K
    (130, 1024, 512, 0, True, 128, 256, 3),      # widest tile, split-K, two token tiles
    (832, 8960, 1536, 1, False, 128, 256, 5),    # down projection, explicit split-K
    # 256-token tiles on SM pairs (cta_group::2): gate on the even CTA, up on the odd one
    (832, 1536, 8960, 2, False, 256, 128, 1),
    (300, 1536, 1536, 1, True, 256, 256, 3),     # split-K, the odd CTA's rows partly past M
    (100, 512, 640, 0, False, 256, 160, 1),      # the odd CTA's rows all past M
    (832, 8960, 1536, 1, False, 256, 192, 6),    # down projection, split-K
    (832, 1536, 2048, 0, True, 256, 128, 1),     # QKV with bias
    (320, 1536, 151936, 0, False, 256, 256, 1),  # internal-node lm_head
    (300, 512, 1024, 2, False, 256, 64, 2),      # SwiGLU split-K on a pair
    # one k chunk per ring slot: an odd number of chunks, or more splits than chunk pairs
    (200, 192, 256, 0, True, 128, 64, 1),
    (300, 320, 512, 1, False, 256, 128, 1),
    (256, 512, 256, 2, False, 128, 64, 8),
])
def test_linear_epilogues_match_fp32(ops, M, K, N, epi, bias, bm, bn, splits):
    """fg_linear against an fp32 torch reference of the same projection and
    epilogue, within the bf16 tolerance (2e-2 of the largest magnitude, 1e-2
    normwise); a second call gives the same bits (split-K adds its partials
    in a fixed order)."""
    g = torch.Generator().manual_seed(M + N + K + 7 * epi)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
    rows = 2 * N if epi == 2 else N
    w = (torch.randn(rows, K, generator=g) * K ** -0.5).to(torch.bfloat16).to(DEV)
    b = torch.randn(N, generator=g).to(torch.bfloat16).to(DEV) if bias else None
    resid = torch.randn(M, N, generator=g).to(torch.bfloat16).to(DEV) if epi == 1 else None
    ref = _linear_ref(x, w, epi, b, resid)
    need = ops.linear_workspace_bytes(M, N, K, epi, bn, splits, bm)
    ws = torch.zeros(need // 4 + 16, dtype=torch.int32, device=DEV) if need else None
    outs = []
    for _ in range(2):
        if epi == 1:
            out = resid.clone()  # the residual add in place, as the verify forward runs it
            got = ops.linear(x, w, bias=b, resid=out, out=out, bm=bm, bn=bn, splits=splits, workspace=ws)
        else:
            out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
            got = ops.linear(x, w, bias=b, out=out, epilogue=epi, bm=bm, bn=bn, splits=splits, workspace=ws)
        outs.append(got)
    torch.cuda.synchronize()
    got = outs[0]
    assert torch.isfinite(got.float()).all()
    d = got.float() - ref
    assert (d.norm() / ref.norm()).item() <= 1e-2
    assert d.abs().max().item() <= 2e-2 * ref.abs().max().item()
    assert torch.equal(outs[1], got)


def test_linear_ring_depths_give_the_same_bits(ops):
    """The ring depth only changes how many k chunks are in flight: 4, 6 and
    8 chunks (2, 3 and 4 two-chunk slots) give identical outputs (the k
    order of the accumulation is the same), for a fused epilogue and a
    split-K tile."""
    g = torch.Generator().manual_seed(3)
    M, K, N = 300, 1024, 512
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(N, K, generator=g) * K ** -0.5).to(torch.bfloat16).to(DEV)
    r = torch.randn(M, N, generator=g).to(torch.bfloat16).to(DEV)
    for bn, splits in ((64, 1), (64, 2)):  # 48 KB two-chunk slots: 4 of them fit
        need = ops.linear_workspace_bytes(M, N, K, 1, bn, splits, 128)
        ws = torch.zeros(need // 4 + 16, dtype=torch.int32, device=DEV) if need else None
        outs = [ops.linear(x, w, resid=r, out=r.clone(), bm=128, bn=bn, splits=splits, stages=st, workspace=ws)
                for st in (4, 6, 8)]
        torch.cuda.synchronize()
        assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2]), (bn, splits)
        ref = _linear_ref(x, w, 1, None, r)
        assert (outs[0].float() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()


def test_linear_rejects_bad_shapes(ops):
    from flashgrpo_b200 import _native

    x = torch.zeros(8, 100, dtype=torch.bfloat16, device=DEV)  # K not a multiple of 64
    w = torch.zeros(16, 100, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(_native.NativeError):
        ops.linear(x, w)
    x = torch.zeros(8, 128, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(16, 128, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(_native.NativeError):
        ops.linear(x, w, bm=128, bn=24, splits=1)  # bn must be a multiple of 16
    need = ops.linear_workspace_bytes(8, 16, 128, 0, 16, 2, 128)
    assert need > 0
    with pytest.raises(ValueError):
        ops.linear(x, w, bm=128, bn=16, splits=2)  # split-K without its workspace


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_norms_and_activations(ops, dtype):
    g = torch.Generator().manual_seed(7)
    x = torch.randn(37, 1536, generator=g).to(dtype).to(DEV)
    w = (torch.rand(1536, generator=g) + 0.5).to(dtype).to(DEV)
    bias = torch.randn(1536, generator=g).to(dtype).to(DEV)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    var = x.float().pow(2).mean(-1, keepdim=True)
    ref = w * (x.float() * torch.rsqrt(var + 1e-6)).to(dtype)
    assert torch.allclose(ops.rmsnorm(x, w, 1e-6).float(), ref.float(), atol=tol, rtol=tol)
    ref_ln = torch.nn.functional.layer_norm(x.float(), (1536,), w.float(), bias.float(), 1e-5)
    assert torch.allclose(ops.layernorm(x, w, bias, 1e-5).float(), ref_ln, atol=tol * 4, rtol=tol)
    gu = torch.randn(37, 2 * 700, generator=g).to(dtype).to(DEV)
    ref_sm = torch.nn.functional.silu(gu[:, :700]) * gu[:, 700:]
    assert torch.allclose(ops.silu_mul(gu).float(), ref_sm.float(), atol=tol, rtol=tol)
    y = torch.randn_like(x)
    assert torch.allclose(ops.silu_residual(x, y).float(), (x + torch.nn.functional.silu(y)).float(), atol=tol,
                          rtol=tol)
    idx = torch.tensor([3, 0, 36, 3], dtype=torch.int32, device=DEV)
    assert torch.equal(ops.gather_rows(x, idx), x[idx.long()])
    # RMSNorm over the model widths (the vectorized kernel up to 8 KB rows)
    for dim, rows in ((256, 9), (3584, 17), (4096, 3)):
        xx = torch.randn(rows, dim, generator=g).to(dtype).to(DEV)
        ww = (torch.rand(dim, generator=g) + 0.5).to(dtype).to(DEV)
        vv = xx.float().pow(2).mean(-1, keepdim=True)
        rr = ww * (xx.float() * torch.rsqrt(vv + 1e-6)).to(dtype)
        assert torch.allclose(ops.rmsnorm(xx, ww, 1e-6).float(), rr.float(), atol=tol, rtol=tol), dim


def test_bounded_wait_times_out_and_context_survives(ops):
    from flashgrpo_b200 import _native

    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    status = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    _native.call("fg_wait_flag", flag.data_ptr(), 20_000_000, status.data_ptr(),
                 torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(status) == _native.FG_ETIMEOUT
    assert _native.read_device_error(clear=True) == _native.FG_ETIMEOUT
    flag.fill_(1)
    _native.call("fg_wait_flag", flag.data_ptr(), 20_000_000, status.data_ptr(),
                 torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(status) == _native.FG_OK
    assert (torch.ones(4, device=DEV) * 2).sum().item() == 8.0

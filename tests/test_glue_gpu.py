"""The fused decoder glue against PyTorch f32 restatements of the same ops
(forward outputs and input gradients), tolerance: max |err| / max |ref|
within bf16 rounding (2e-2)."""
from __future__ import annotations

import pytest

TOL = 2e-2


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()


@pytest.mark.gpu
@pytest.mark.parametrize("rows,hidden", [(1, 8), (37, 896), (4096, 4096), (3, 14336)])
def test_rms_norm(cuda, rows, hidden):
    import torch

    from torobi_b200 import glue

    torch.manual_seed(rows)
    x = (torch.randn(rows, hidden, device=cuda) * 3).bfloat16().requires_grad_()
    w = (torch.rand(hidden, device=cuda) + 0.5).bfloat16()
    dy = torch.randn(rows, hidden, device=cuda).bfloat16()
    y = glue.rms_norm(x, w, 1e-6)
    (dx,) = torch.autograd.grad(y, x, dy)
    xf = x.detach().float().requires_grad_()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    (dref,) = torch.autograd.grad(ref, xf, dy.float())
    assert _rel(y, ref) < TOL
    assert _rel(dx, dref) < TOL


@pytest.mark.gpu
@pytest.mark.parametrize("rows,hidden", [(1, 8), (37, 896), (4096, 4096), (3, 14336)])
def test_add_rms_norm(cuda, rows, hidden):
    """s = x + res and its norm in one kernel: s and y bit-equal to the
    separate bf16 add and rms_norm; the gradients of x and res (the norm's
    backward with the stream's gradient added inside) against f32, and the
    stream's gradient alone passed through when the norm output is unused."""
    import torch

    from torobi_b200 import glue

    torch.manual_seed(rows + 1)
    x = (torch.randn(rows, hidden, device=cuda) * 3).bfloat16().requires_grad_()
    res = torch.randn(rows, hidden, device=cuda).bfloat16().requires_grad_()
    w = (torch.rand(hidden, device=cuda) + 0.5).bfloat16()
    ds = torch.randn(rows, hidden, device=cuda).bfloat16()
    dy = torch.randn(rows, hidden, device=cuda).bfloat16()
    s, y = glue.add_rms_norm(x, res, w, 1e-6)
    s_sep = x.detach() + res.detach()
    assert torch.equal(s.detach().view(torch.int16), s_sep.view(torch.int16))
    y_sep = glue.rms_norm(s_sep, w, 1e-6)
    assert torch.equal(y.detach().view(torch.int16), y_sep.view(torch.int16))
    dx, dres = torch.autograd.grad((s, y), (x, res), (ds, dy))
    sf = s_sep.float().requires_grad_()
    ref = sf * torch.rsqrt(sf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    (dref,) = torch.autograd.grad(ref, sf, dy.float())
    dref = dref + ds.float()
    assert _rel(dx, dref) < TOL and torch.equal(dx, dres)
    s2, _ = glue.add_rms_norm(x, res, w, 1e-6)
    (dx2,) = torch.autograd.grad(s2, x, ds)
    assert torch.equal(dx2, ds)


@pytest.mark.gpu
@pytest.mark.parametrize("b,s,h,d", [(2, 16, 4, 64), (1, 2048, 8, 128), (3, 7, 14, 64)])
def test_rope_and_its_inverse(cuda, b, s, h, d):
    import torch

    from torobi_b200 import glue
    from torobi_b200.model import apply_rope, rope_tables

    torch.manual_seed(s)
    cos, sin = rope_tables(s, d, 5e5, cuda)
    x = torch.randn(b, s, h, d, device=cuda).bfloat16().requires_grad_()
    y = glue.rope(x, cos, sin)
    ref = apply_rope(x.detach().float().transpose(1, 2), cos, sin).transpose(1, 2)
    assert _rel(y, ref) < TOL
    dy = torch.randn_like(y)
    (dx,) = torch.autograd.grad(y, x, dy)
    xf = x.detach().float().transpose(1, 2).requires_grad_()
    (dref,) = torch.autograd.grad(apply_rope(xf, cos, sin), xf, dy.float().transpose(1, 2))
    assert _rel(dx, dref.transpose(1, 2)) < TOL


@pytest.mark.gpu
@pytest.mark.parametrize("n", [8, 4864 * 3, 8192 * 14336 // 64])
def test_swiglu(cuda, n):
    import torch
    import torch.nn.functional as F

    from torobi_b200 import glue

    torch.manual_seed(0)
    g = (torch.randn(n, device=cuda) * 2).bfloat16().requires_grad_()
    u = torch.randn(n, device=cuda).bfloat16().requires_grad_()
    a = glue.swiglu(g, u)
    da = torch.randn(n, device=cuda).bfloat16()
    dg, du = torch.autograd.grad(a, (g, u), da)
    gf = g.detach().float().requires_grad_()
    uf = u.detach().float().requires_grad_()
    ref = F.silu(gf) * uf
    dgr, dur = torch.autograd.grad(ref, (gf, uf), da.float())
    assert _rel(a, ref) < TOL
    assert _rel(dg, dgr) < TOL
    assert _rel(du, dur) < TOL

"""Fused decoder glue as differentiable ops: RMSNorm, rotary embedding and
SwiGLU, each one sm_100a kernel forward and one backward (csrc/glue.cu).

RMSNorm is ``x * rsqrt(mean(x^2) + eps) * w`` (engine/src/interp.rs:312-319),
with a frozen gain; RoPE rotates the first half of each head against the
second (engine/src/interp.rs:350-388); SwiGLU is ``(g * sigmoid(g)) * u``
(lib/torobi/models/llama.rb:320-327).
"""
from __future__ import annotations

import ctypes

import torch

from .ops import _launch, _need_cuda, _ptr, _stream
from ._lib import check, lib


def _bf16_contig(name: str, t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bfloat16, got {t.dtype}")
    return t.contiguous()


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        _need_cuda("rms_norm", x=x, w=w)
        x = _bf16_contig("x", x)
        w = _bf16_contig("w", w)
        h = x.shape[-1]
        rows = x.numel() // h
        y = torch.empty_like(x)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        _launch("rmsnorm", lambda: lib().tq_rmsnorm_fwd(_ptr(x), _ptr(w), rows, h, float(eps),
                                                         _ptr(y), _ptr(rstd), _stream()))
        ctx.save_for_backward(x, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dy = dy.contiguous()
        h = x.shape[-1]
        rows = x.numel() // h
        dx = torch.empty_like(x)
        _launch("rmsnorm", lambda: lib().tq_rmsnorm_bwd(_ptr(x), _ptr(w), _ptr(rstd), _ptr(dy),
                                                         None, rows, h, _ptr(dx), _stream()))
        return dx, None, None


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm over the last axis; differentiable wrt x (the gain is frozen)."""
    return _RMSNorm.apply(x, w, eps)


class _AddRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, res, w, eps):
        _need_cuda("add_rms_norm", x=x, res=res, w=w)
        x = _bf16_contig("x", x)
        res = _bf16_contig("res", res)
        w = _bf16_contig("w", w)
        if res.shape != x.shape:
            raise ValueError(f"[add_rms_norm] res {tuple(res.shape)} must match x "
                             f"{tuple(x.shape)}")
        h = x.shape[-1]
        rows = x.numel() // h
        s = torch.empty_like(x)
        y = torch.empty_like(x)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        _launch("rmsnorm", lambda: lib().tq_add_rmsnorm_fwd(
            _ptr(x), _ptr(res), _ptr(w), rows, h, float(eps), _ptr(s), _ptr(y), _ptr(rstd),
            _stream()))
        ctx.save_for_backward(s, w, rstd)
        ctx.set_materialize_grads(False)
        return s, y

    @staticmethod
    def backward(ctx, ds, dy):
        s, w, rstd = ctx.saved_tensors
        if dy is None:
            return ds, ds, None, None
        dy = dy.contiguous()
        ds = ds.contiguous() if ds is not None else None
        h = s.shape[-1]
        rows = s.numel() // h
        dx = torch.empty_like(s)
        _launch("rmsnorm", lambda: lib().tq_rmsnorm_bwd(
            _ptr(s), _ptr(w), _ptr(rstd), _ptr(dy), _ptr(ds) if ds is not None else None, rows, h,
            _ptr(dx), _stream()))
        return dx, dx, None, None


def add_rms_norm(x: torch.Tensor, res: torch.Tensor, w: torch.Tensor, eps: float):
    """``(s, rms_norm(s, w, eps))`` with ``s = x + res`` in bf16: a pre-norm
    block's residual add and the norm after it in one kernel; its backward
    adds the residual stream's gradient inside the norm's (one kernel)."""
    return _AddRMSNorm.apply(x, res, w, eps)


class _RoPE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cos, sin, seq):
        _need_cuda("rope", x=x, cos=cos, sin=sin)
        x = _bf16_contig("x", x)
        tokens, heads, dim = x.shape[0] * x.shape[1], x.shape[2], x.shape[3]
        y = torch.empty_like(x)
        _launch("rope", lambda: lib().tq_rope(_ptr(x), tokens, heads, dim, seq, _ptr(cos),
                                               _ptr(sin), 0, _ptr(y), _stream()))
        ctx.save_for_backward(cos, sin)
        ctx.seq = seq
        return y

    @staticmethod
    def backward(ctx, dy):
        cos, sin = ctx.saved_tensors
        dy = dy.contiguous()
        tokens, heads, dim = dy.shape[0] * dy.shape[1], dy.shape[2], dy.shape[3]
        dx = torch.empty_like(dy)
        _launch("rope", lambda: lib().tq_rope(_ptr(dy), tokens, heads, dim, ctx.seq, _ptr(cos),
                                               _ptr(sin), 1, _ptr(dx), _stream()))
        return dx, None, None, None


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [batch, seq, heads, dim] bf16; cos/sin [seq, dim/2] f32."""
    return _RoPE.apply(x, cos.contiguous(), sin.contiguous(), x.shape[1])


def attention_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                      scale: float | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Grouped-query scaled dot-product attention (engine/src/interp.rs:405-432).

    q [batch, seq, heads, dim], k/v [batch, seq, kv_heads, dim] bf16 (dim 64
    or 128).  Returns o in q's layout and lse [batch, heads, seq] f32 (the
    natural-log log-sum-exp of each query row's scaled scores)."""
    _need_cuda("attention", q=q, k=k, v=v)
    q = _bf16_contig("q", q)
    k = _bf16_contig("k", k)
    v = _bf16_contig("v", v)
    if q.dim() != 4 or k.shape != v.shape or k.dim() != 4:
        raise ValueError(f"[attention] q {tuple(q.shape)}, k {tuple(k.shape)}, v "
                         f"{tuple(v.shape)}: want [batch, seq, heads, dim] and equal k/v")
    b, s, h, d = q.shape
    if k.shape[0] != b or k.shape[1] != s or k.shape[3] != d:
        raise ValueError(f"[attention] k {tuple(k.shape)} does not match q {tuple(q.shape)}")
    hk = k.shape[2]
    sc = float(scale) if scale is not None else d ** -0.5
    o = torch.empty_like(q)
    lse = torch.empty(b, h, s, dtype=torch.float32, device=q.device)
    _launch("attention", lambda: lib().tq_attention_fwd(
        _ptr(q), _ptr(k), _ptr(v), b, s, h, hk, d, sc, int(bool(causal)), _ptr(o), _ptr(lse),
        _stream()))
    return o, lse


def attention_backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor,
                       do: torch.Tensor, lse: torch.Tensor, causal: bool = True,
                       scale: float | None = None):
    """dq, dk, dv of ``attention_forward`` given the upstream gradient do
    (q's layout) and the forward's o and lse."""
    _need_cuda("attention", q=q, k=k, v=v, o=o, do=do, lse=lse)
    q, k, v, o = (_bf16_contig(n, t) for n, t in (("q", q), ("k", k), ("v", v), ("o", o)))
    do = _bf16_contig("do", do)
    if o.shape != q.shape or do.shape != q.shape:
        raise ValueError("[attention] o and do must have q's shape")
    b, s, h, d = q.shape
    hk = k.shape[2]
    if lse.dtype != torch.float32 or tuple(lse.shape) != (b, h, s):
        raise ValueError(f"[attention] lse must be f32 [{b}, {h}, {s}]")
    lse = lse.contiguous()
    sc = float(scale) if scale is not None else d ** -0.5
    nbytes = ctypes.c_size_t()
    check(lib().tq_attention_bwd_workspace_bytes(b, s, h, ctypes.byref(nbytes)))
    ws = torch.empty(max(1, nbytes.value), dtype=torch.uint8, device=q.device)
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    _launch("attention", lambda: lib().tq_attention_bwd(
        _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(do), _ptr(lse), b, s, h, hk, d, sc,
        int(bool(causal)), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(ws), nbytes.value, _stream()))
    return dq, dk, dv


class _Attention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale):
        o, lse = attention_forward(q, k, v, causal, scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal, ctx.scale = causal, scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = attention_backward(q, k, v, o, do, lse, ctx.causal, ctx.scale)
        return dq, dk, dv, None, None


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
              scale: float | None = None) -> torch.Tensor:
    """Differentiable grouped-query attention: q [batch, seq, heads, dim],
    k/v [batch, seq, kv_heads, dim] bf16, output in q's layout; the scale
    defaults to dim^-1/2 (engine/src/interp.rs:405-432)."""
    return _Attention.apply(q, k, v, causal, scale)


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, g, u):
        _need_cuda("swiglu", g=g, u=u)
        g = _bf16_contig("g", g)
        u = _bf16_contig("u", u)
        a = torch.empty_like(g)
        _launch("swiglu", lambda: lib().tq_swiglu_fwd(_ptr(g), _ptr(u), g.numel(), _ptr(a),
                                                       _stream()))
        ctx.save_for_backward(g, u)
        return a

    @staticmethod
    def backward(ctx, da):
        g, u = ctx.saved_tensors
        da = da.contiguous()
        dg = torch.empty_like(g)
        du = torch.empty_like(u)
        _launch("swiglu", lambda: lib().tq_swiglu_bwd(_ptr(g), _ptr(u), _ptr(da), g.numel(),
                                                       _ptr(dg), _ptr(du), _stream()))
        return dg, du


def swiglu(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """(g * sigmoid(g)) * u."""
    return _SwiGLU.apply(g, u)


class _CrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z, targets, inplace):
        _need_cuda("cross_entropy", z=z, targets=targets)
        z = _bf16_contig("logits", z)
        vocab = z.shape[-1]
        rows = z.numel() // vocab if vocab else 0
        t = targets.reshape(-1).to(torch.int64).contiguous()
        if t.numel() != rows:
            raise ValueError(f"targets hold {t.numel()} positions, logits {rows}")
        lse = torch.empty(rows, dtype=torch.float32, device=z.device)
        loss = torch.empty(rows, dtype=torch.float32, device=z.device)
        _launch("cross_entropy", lambda: lib().tq_cross_entropy_fwd(
            _ptr(z), _ptr(t), rows, vocab, vocab, _ptr(lse), _ptr(loss), _stream()))
        ctx.save_for_backward(z, t, lse)
        ctx.inplace = inplace
        return loss.view(z.shape[:-1])

    @staticmethod
    def backward(ctx, dloss):
        z, t, lse = ctx.saved_tensors
        vocab = z.shape[-1]
        rows = z.numel() // vocab
        dl = dloss.reshape(-1).float().contiguous()
        dz = z if ctx.inplace else torch.empty_like(z)
        _launch("cross_entropy", lambda: lib().tq_cross_entropy_bwd(
            _ptr(z), _ptr(t), _ptr(lse), rows, vocab, vocab, _ptr(dl), 1.0, _ptr(dz), _stream()))
        return dz, None, None


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor,
                  inplace: bool = False) -> torch.Tensor:
    """Per-position ``logsumexp(logits) - logits[target]`` in f32 (no
    reduction, as the reference's loss node), logits bf16 [..., vocab].
    ``inplace=True`` writes the gradient over the logits in backward (no
    second [rows, vocab] buffer); the graph then cannot be run backward twice."""
    return _CrossEntropy.apply(logits, targets, inplace)

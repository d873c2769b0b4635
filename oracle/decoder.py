"""CPU restatement of one QLoRA training step of the Llama-shaped decoder
(test infrastructure only: the CPU baseline of the benchmark and the
reference arm time it; nothing in ``torobi_b200`` imports it).

numpy f32 arithmetic on bf16 values, every op's output rounded to bf16 as the
model's bf16 activations are, the quantized linears through the C oracle
(``oracle.qlora_linear_fwd/bwd``, ``oracle.qmm_fwd/dx``).  Each piece follows
the reference's rule for it:

* the pre-norm block ``x += attn(norm(x)); x += mlp(norm(x))``
  (lib/torobi/models/llama.rb:263-267), its projections q/k/v/o
  (:297-315) and gate/up/down (:320-327);
* RMSNorm ``x * rsqrt(mean(x^2) + eps) * w`` (engine/src/interp.rs:312-319);
* RoPE, the first half of each head rotated against the second by
  ``p / theta^(2i/d)`` (engine/src/interp.rs:350-388);
* causal scaled-dot-product attention with grouped KV heads
  (engine/src/interp.rs:405-432), softmax in f32;
* SwiGLU ``(g * sigmoid(g)) * u`` (lib/torobi/models/llama.rb:320-327);
* the head ``h . E^T`` and the per-position f32 cross-entropy
  (engine/src/interp.rs:440-444);
* AdamW on the adapter (engine/src/optimizer.rs:305-352).
The backward is the VJP MLX derives for that graph (engine/src/executor.rs:163-191):
adapter gradients and the input gradient; the base weights get none.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from . import oracle as O

F32 = np.float32


def rb(x):
    """Round f32 values to bf16 (the model stores its activations in bf16)."""
    return O.round_bf16(np.asarray(x, F32))


# ------------------------------------------------------------- pieces ------

def rms_norm(x, w, eps):
    """engine/src/interp.rs:312-319; returns (y, rstd)."""
    rstd = (1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True, dtype=F32) + F32(eps))).astype(F32)
    return rb(x * rstd * w), rstd


def rms_norm_vjp(x, w, rstd, dy):
    """d/dx of x * rstd * w: rstd*dy*w - x * rstd^3 * mean(dy*w*x)."""
    dyw = dy * w
    m = np.mean(dyw * x, axis=-1, keepdims=True, dtype=F32)
    return rb(rstd * dyw - x * (rstd ** 3) * m)


def rope_tables(seq, dim, theta):
    half = dim // 2
    p = np.arange(seq, dtype=F32)[:, None]
    i = np.arange(half, dtype=F32)[None, :]
    ang = p / np.power(F32(theta), (F32(2.0) * i / F32(dim)).astype(F32)).astype(F32)
    return np.cos(ang).astype(F32), np.sin(ang).astype(F32)


def rope(x, cos, sin, inverse=False):
    """x [T, H, D] (position = row); engine/src/interp.rs:350-388.  The inverse
    rotation is the VJP."""
    half = x.shape[-1] // 2
    a, b = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], (-sin if inverse else sin)[:, None, :]
    return rb(np.concatenate([a * c - b * s, b * c + a * s], axis=-1))


def attention(q, k, v):
    """Causal GQA attention over one sequence, q [T, Hq, D], k/v [T, Hkv, D]
    (engine/src/interp.rs:405-432).  Returns (o [T, Hq, D], probs)."""
    T, Hq, D = q.shape
    rep = Hq // k.shape[1]
    kk = np.repeat(k, rep, axis=1).transpose(1, 0, 2)  # [Hq, T, D]
    vv = np.repeat(v, rep, axis=1).transpose(1, 0, 2)
    qq = q.transpose(1, 0, 2)
    s = (qq @ kk.transpose(0, 2, 1)) * F32(1.0 / math.sqrt(D))
    s = s + np.triu(np.full((T, T), -np.inf, F32), 1)[None]
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s).astype(F32)
    p /= p.sum(-1, keepdims=True)
    o = (p @ vv).transpose(1, 0, 2)
    return rb(o), p


def attention_vjp(q, k, v, p, do):
    T, Hq, D = q.shape
    hk = k.shape[1]
    rep = Hq // hk
    kk = np.repeat(k, rep, axis=1).transpose(1, 0, 2)
    vv = np.repeat(v, rep, axis=1).transpose(1, 0, 2)
    qq = q.transpose(1, 0, 2)
    dd = do.transpose(1, 0, 2)
    dv = p.transpose(0, 2, 1) @ dd                      # [Hq, T, D]
    dp = dd @ vv.transpose(0, 2, 1)
    ds = p * (dp - np.sum(dp * p, -1, keepdims=True)) * F32(1.0 / math.sqrt(D))
    dq = ds @ kk
    dk = ds.transpose(0, 2, 1) @ qq
    dk = dk.reshape(hk, rep, T, D).sum(1)
    dv = dv.reshape(hk, rep, T, D).sum(1)
    return (rb(dq.transpose(1, 0, 2)), rb(dk.transpose(1, 0, 2)), rb(dv.transpose(1, 0, 2)))


def swiglu(g, u):
    sg = (1.0 / (1.0 + np.exp(-g))).astype(F32)
    return rb(g * sg * u)


def swiglu_vjp(g, u, da):
    sg = (1.0 / (1.0 + np.exp(-g))).astype(F32)
    silu = g * sg
    du = da * silu
    dg = da * u * (sg * (1.0 + g * (1.0 - sg)))
    return rb(dg), rb(du)


# ---------------------------------------------------------- the block ------

@dataclass
class Linear:
    codes: np.ndarray
    scales: np.ndarray
    biases: np.ndarray
    a: np.ndarray | None = None  # f32 [r, d_in] (bf16 values)
    b: np.ndarray | None = None  # f32 [d_out, r]
    ga: np.ndarray | None = None
    gb: np.ndarray | None = None


@dataclass
class Block:
    input_norm: np.ndarray
    post_norm: np.ndarray
    lin: dict = field(default_factory=dict)


@dataclass
class Shape:
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    rope_theta: float
    rms_eps: float
    bits: int
    group: int
    rank: int
    alpha: float
    targets: tuple


def make_block(shape: Shape, rng) -> Block:
    """A block's quantized linears (N(0, 0.02) weights through the oracle's
    quantize) and adapters (A ~ N(0, 1/8), B ~ N(0, 0.01), as bf16 values)."""
    h, i = shape.hidden, shape.intermediate
    q, kv = shape.heads * shape.head_dim, shape.kv_heads * shape.head_dim
    shapes = {"q_proj": (q, h), "k_proj": (kv, h), "v_proj": (kv, h), "o_proj": (h, q),
              "gate_proj": (i, h), "up_proj": (i, h), "down_proj": (h, i)}
    blk = Block(np.ones(h, F32), np.ones(h, F32))
    for name, (o, n) in shapes.items():
        c, s, b = O.quantize(O.normal_bf16(rng, (o, n), 0.02), shape.bits, shape.group)
        L = Linear(c, s, b)
        if name in shape.targets:
            L.a = O.f32_from_bf16(O.normal_bf16(rng, (shape.rank, n), 0.125))
            L.b = O.f32_from_bf16(O.normal_bf16(rng, (o, shape.rank), 0.01))
            L.ga = np.zeros_like(L.a)
            L.gb = np.zeros_like(L.b)
        blk.lin[name] = L
    return blk


def _lin_fwd(shape, L, x):
    if L.a is None:
        return rb(O.qmm_fwd(O.bf16_from_f32(x), L.codes, L.scales, L.biases, shape.bits,
                            shape.group))
    y, _ = O.qlora_linear_fwd(x, L.codes, L.scales, L.biases, L.a, L.b,
                              shape.alpha / shape.rank, shape.bits, shape.group)
    return y


def _lin_bwd(shape, L, x, dy):
    if L.a is None:
        return rb(O.qmm_dx(O.bf16_from_f32(dy), L.codes, L.scales, L.biases, shape.bits,
                           shape.group))
    dx, da, db = O.qlora_linear_bwd(x, dy, L.codes, L.scales, L.biases, L.a, L.b,
                                    shape.alpha / shape.rank, shape.bits, shape.group)
    L.ga += da
    L.gb += db
    return dx


def block_step(shape: Shape, blk: Block, x, dout_fn):
    """Forward of one block on x [T, hidden] (one sequence), then its VJP with
    the output gradient ``dout_fn(out)``; accumulates the adapter gradients
    into the block and returns (out, dx)."""
    T = x.shape[0]
    cos, sin = rope_tables(T, shape.head_dim, shape.rope_theta)
    hq, hk, d = shape.heads, shape.kv_heads, shape.head_dim
    h1, r1 = rms_norm(x, blk.input_norm, shape.rms_eps)
    q = rope(_lin_fwd(shape, blk.lin["q_proj"], h1).reshape(T, hq, d), cos, sin)
    k = rope(_lin_fwd(shape, blk.lin["k_proj"], h1).reshape(T, hk, d), cos, sin)
    v = _lin_fwd(shape, blk.lin["v_proj"], h1).reshape(T, hk, d)
    att, probs = attention(q, k, v)
    att2 = att.reshape(T, hq * d)
    x2 = rb(x + _lin_fwd(shape, blk.lin["o_proj"], att2))
    h2, r2 = rms_norm(x2, blk.post_norm, shape.rms_eps)
    g = _lin_fwd(shape, blk.lin["gate_proj"], h2)
    u = _lin_fwd(shape, blk.lin["up_proj"], h2)
    a = swiglu(g, u)
    out = rb(x2 + _lin_fwd(shape, blk.lin["down_proj"], a))

    dout = dout_fn(out)
    da = _lin_bwd(shape, blk.lin["down_proj"], a, dout)
    dg, du = swiglu_vjp(g, u, da)
    dh2 = rb(_lin_bwd(shape, blk.lin["gate_proj"], h2, dg) +
             _lin_bwd(shape, blk.lin["up_proj"], h2, du))
    dx2 = rb(dout + rms_norm_vjp(x2, blk.post_norm, r2, dh2))
    datt = _lin_bwd(shape, blk.lin["o_proj"], att2, dx2).reshape(T, hq, d)
    dq, dk, dv = attention_vjp(q, k, v, probs, datt)
    dq = rope(dq, cos, sin, inverse=True).reshape(T, hq * d)
    dk = rope(dk, cos, sin, inverse=True).reshape(T, hk * d)
    dh1 = rb(_lin_bwd(shape, blk.lin["q_proj"], h1, dq) +
             _lin_bwd(shape, blk.lin["k_proj"], h1, dk) +
             _lin_bwd(shape, blk.lin["v_proj"], h1, dv.reshape(T, hk * d)))
    dx = rb(dx2 + rms_norm_vjp(x, blk.input_norm, r1, dh1))
    return out, dx


def head_loss_step(h, head, targets):
    """Logits ``h . head^T`` in bf16, the mean f32 cross-entropy over the
    positions and its VJP back to h.  Returns (loss, dh)."""
    z = rb(h @ head.T)
    loss = O.cross_entropy(z, targets)
    dz = rb(O.cross_entropy_vjp(z, targets, np.full(len(targets), 1.0 / len(targets), F32)))
    return float(loss.mean()), rb(dz @ head)


def adamw_block(blk: Block, t: int, lr: float = 1e-4):
    """AdamW over a block's adapters (moments kept on the Linear)."""
    for L in blk.lin.values():
        if L.a is None:
            continue
        for name in ("a", "b"):
            p = getattr(L, name)
            g = getattr(L, "g" + name)
            m = getattr(L, "m" + name, None)
            v = getattr(L, "v" + name, None)
            if m is None:
                m = np.zeros_like(p)
                v = np.zeros_like(p)
            p2, m2, v2 = O.adamw_step(p, g, m, v, t, lr)
            setattr(L, name, p2)
            setattr(L, "m" + name, m2)
            setattr(L, "v" + name, v2)
            g[...] = 0.0

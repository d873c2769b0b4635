"""The tensor-core attention (csrc/attn.cu) against a PyTorch f32 restatement
of grouped-query scaled dot-product attention with a causal mask (the
reference's node: engine/src/interp.rs:405-432, MLX's fused SDPA).

Tolerances: outputs and input gradients max |err| / max |ref| <= 1e-2 (bf16
operands, f32 accumulation, probabilities rounded to bf16 before P V); the
log-sum-exp within 2e-3 absolute (it is f32 from unrounded probabilities).
"""
from __future__ import annotations

import pytest

TOL = 1e-2
LSE_TOL = 2e-3


def _rel(a, b):
    """max |err| / max |ref|, the denominator floored at 1e-3: a gradient
    that is exactly zero in exact arithmetic (one position: softmax is 1, so
    dq = dk = 0) comes out as rounding noise of order 1e-7."""
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-3)).item()


def reference_attention(q, k, v, causal: bool, scale: float):
    """o [B, S, H, D] and lse [B, H, S] in f32 from bf16 q/k/v (k/v heads
    shared by heads // kv_heads consecutive query heads)."""
    import torch

    b, s, h, d = q.shape
    g = h // k.shape[2]
    qf = q.float().transpose(1, 2)
    kf = k.float().transpose(1, 2).repeat_interleave(g, dim=1)
    vf = v.float().transpose(1, 2).repeat_interleave(g, dim=1)
    outs, lses = [], []
    for hi in range(h):  # one head at a time keeps the [S, S] scores small
        sc = (qf[:, hi] @ kf[:, hi].transpose(-1, -2)) * scale
        if causal:
            mask = torch.ones(s, s, dtype=torch.bool, device=q.device).triu(1)
            sc = sc.masked_fill(mask, float("-inf"))
        lses.append(torch.logsumexp(sc, -1))
        outs.append(torch.softmax(sc, -1) @ vf[:, hi])
    return torch.stack(outs, 2), torch.stack(lses, 1)


def _inputs(cuda, seed, b, s, h, hk, d, q_gain=1.0):
    import torch

    g = torch.Generator(device=cuda)
    g.manual_seed(seed)
    q = (torch.randn(b, s, h, d, device=cuda, generator=g) * q_gain).bfloat16()
    k = torch.randn(b, s, hk, d, device=cuda, generator=g).bfloat16()
    v = torch.randn(b, s, hk, d, device=cuda, generator=g).bfloat16()
    return q, k, v


CASES = [
    # (batch, seq, heads, kv_heads, dim, causal)
    (2, 256, 4, 2, 64, True),
    (1, 300, 4, 1, 128, True),      # ragged: the last tiles are partly past seq
    (2, 200, 2, 2, 128, False),     # no mask, ragged
    (1, 1, 2, 1, 64, True),         # one position
    (2, 512, 14, 2, 64, True),      # Qwen2.5-0.5B heads (14 over 2, dim 64), seq 512
    (1, 2048, 32, 8, 128, True),    # Llama-3-8B heads (32 over 8, dim 128), seq 2048
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: "b{}_s{}_h{}_{}_d{}_{}".format(
    *c[:5], "causal" if c[5] else "full"))
def test_attention_forward(cuda, case):
    from torobi_b200 import glue

    b, s, h, hk, d, causal = case
    q, k, v = _inputs(cuda, 11 + s, b, s, h, hk, d)
    scale = d ** -0.5
    o, lse = glue.attention_forward(q, k, v, causal, scale)
    o_ref, lse_ref = reference_attention(q, k, v, causal, scale)
    assert _rel(o, o_ref) <= TOL
    assert (lse - lse_ref).abs().max().item() <= LSE_TOL * max(1.0, lse_ref.abs().max().item())


@pytest.mark.gpu
def test_attention_forward_large_scores(cuda):
    """Scores spanning far more than 2^8 within a row: the running maximum
    moves and the accumulator is rescaled in tensor memory."""
    from torobi_b200 import glue

    q, k, v = _inputs(cuda, 5, 1, 640, 4, 2, 128, q_gain=12.0)
    o, lse = glue.attention_forward(q, k, v, True, 128 ** -0.5)
    o_ref, lse_ref = reference_attention(q, k, v, True, 128 ** -0.5)
    assert _rel(o, o_ref) <= TOL
    assert (lse - lse_ref).abs().max().item() <= LSE_TOL * max(1.0, lse_ref.abs().max().item())


@pytest.mark.gpu
def test_attention_argument_errors(cuda):
    import torch

    from torobi_b200 import TqError, glue

    q = torch.zeros(1, 8, 4, 96, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(TqError, match="head dim"):
        glue.attention_forward(q, q[:, :, :2], q[:, :, :2])
    q = torch.zeros(1, 8, 3, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(TqError, match="multiple of kv_heads"):
        glue.attention_forward(q, q[:, :, :2].contiguous(), q[:, :, :2].contiguous())


def _reference_grads(q, k, v, do, causal, scale):
    import torch

    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    b, s, h, d = q.shape
    g = h // k.shape[2]
    kk = kf.transpose(1, 2).repeat_interleave(g, dim=1)
    vv = vf.transpose(1, 2).repeat_interleave(g, dim=1)
    sc = (qf.transpose(1, 2) @ kk.transpose(-1, -2)) * scale
    if causal:
        mask = torch.ones(s, s, dtype=torch.bool, device=q.device).triu(1)
        sc = sc.masked_fill(mask, float("-inf"))
    o = (torch.softmax(sc, -1) @ vv).transpose(1, 2)
    return torch.autograd.grad(o, (qf, kf, vf), do.float())


BWD_CASES = [
    (2, 256, 4, 2, 64, True),
    (1, 300, 4, 1, 128, True),      # ragged
    (2, 200, 2, 2, 128, False),     # no mask, ragged
    (1, 1, 2, 1, 64, True),
    (2, 512, 14, 2, 64, True),      # Qwen2.5-0.5B heads
    (1, 1024, 32, 8, 128, True),    # Llama-3-8B heads
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", BWD_CASES, ids=lambda c: "b{}_s{}_h{}_{}_d{}_{}".format(
    *c[:5], "causal" if c[5] else "full"))
def test_attention_backward(cuda, case):
    """dq, dk, dv through the autograd op against autograd of the f32
    restatement (dk/dv summed over the query heads of each group)."""
    import torch

    from torobi_b200 import glue

    b, s, h, hk, d, causal = case
    q, k, v = _inputs(cuda, 21 + s, b, s, h, hk, d)
    g = torch.Generator(device=cuda)
    g.manual_seed(3 + s)
    do = torch.randn(b, s, h, d, device=cuda, generator=g).bfloat16()
    qq, kk, vv = (t.clone().requires_grad_() for t in (q, k, v))
    o = glue.attention(qq, kk, vv, causal)
    dq, dk, dv = torch.autograd.grad(o, (qq, kk, vv), do)
    rq, rk, rv = _reference_grads(q, k, v, do, causal, d ** -0.5)
    for name, got, ref in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
        assert _rel(got, ref) <= TOL, f"{name}: {_rel(got, ref):.3e}"


@pytest.mark.gpu
def test_attention_backward_is_deterministic(cuda):
    import torch

    from torobi_b200 import glue

    q, k, v = _inputs(cuda, 9, 2, 384, 8, 2, 128)
    do = torch.randn_like(q)
    o, lse = glue.attention_forward(q, k, v, True)
    first = glue.attention_backward(q, k, v, o, do, lse, True)
    again = glue.attention_backward(q, k, v, o, do, lse, True)
    for a, b_ in zip(first, again):
        assert torch.equal(a, b_)


@pytest.mark.gpu
def test_attention_random_shapes(cuda):
    """Seeded random shapes -- sequence lengths that end anywhere inside a
    64- or 128-row tile, group sizes 1 to 8, both head dims, masked and not
    -- forward and backward against the f32 restatement."""
    import random

    import torch

    from torobi_b200 import glue

    rnd = random.Random(20261202)
    for trial in range(12):
        d = rnd.choice((64, 128))
        hk = rnd.choice((1, 2, 4))
        h = hk * rnd.choice((1, 2, 4, 8))
        b = rnd.randint(1, 3)
        s = rnd.randint(1, 700)
        causal = rnd.random() < 0.75
        q, k, v = _inputs(cuda, 100 + trial, b, s, h, hk, d)
        scale = d ** -0.5
        o, lse = glue.attention_forward(q, k, v, causal, scale)
        o_ref, lse_ref = reference_attention(q, k, v, causal, scale)
        case = (b, s, h, hk, d, causal)
        assert _rel(o, o_ref) <= TOL, case
        assert (lse - lse_ref).abs().max().item() <= LSE_TOL * max(1.0, lse_ref.abs().max().item()), case
        do = torch.randn_like(q)
        qq, kk, vv = (t.clone().requires_grad_() for t in (q, k, v))
        dq, dk, dv = torch.autograd.grad(glue.attention(qq, kk, vv, causal), (qq, kk, vv), do)
        rq, rk, rv = _reference_grads(q, k, v, do, causal, scale)
        for name, got, ref in (("dq", dq, rq), ("dk", dk, rk), ("dv", dv, rv)):
            assert _rel(got, ref) <= TOL, (case, name, _rel(got, ref))

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
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-30)).item()


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

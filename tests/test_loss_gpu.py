"""Parity of the fused cross-entropy (forward per-position loss and its VJP)
with the oracle's f32 restatement of the reference's loss node
(engine/src/interp.rs:434-444): logsumexp(logits) - logits[target].

Tolerances: loss within 1e-5 relative (f32 sums in a different order, fast
exp); gradient within one bf16 rounding (2^-8 relative) plus 1e-6 of the
row's largest entry.
"""
from __future__ import annotations

import numpy as np
import pytest

from _util import dev_bf16, host_bf16

# (rows, vocab, logit std): vocab % 8 == 0 takes 16-byte loads, the others
# the element path; the last is the Llama-3 vocabulary.
CASES = [
    (64, 1024, 1.0),
    (37, 1000, 3.0),
    (5, 13, 1.0),
    (16, 32000, 8.0),
    (4, 128256, 2.0),
]


def _inputs(oracle, rng, rows, vocab, std):
    z = oracle.normal_bf16(rng, (rows, vocab), std)
    t = rng.integers(0, vocab, size=rows, dtype=np.int64)
    return z, t


def _run(cuda, z_bits, t, dloss=None, inplace=False):
    import torch

    from torobi_b200._lib import check, lib

    rows, vocab = z_bits.shape
    z = dev_bf16(z_bits, cuda)
    tt = torch.from_numpy(t).to(cuda)
    lse = torch.empty(rows, dtype=torch.float32, device=cuda)
    loss = torch.empty(rows, dtype=torch.float32, device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    check(lib().tq_cross_entropy_fwd(z.data_ptr(), tt.data_ptr(), rows, vocab, vocab,
                                     lse.data_ptr(), loss.data_ptr(), s))
    dl = None if dloss is None else torch.from_numpy(dloss).to(cuda)
    dz = z if inplace else torch.empty_like(z)
    check(lib().tq_cross_entropy_bwd(z.data_ptr(), tt.data_ptr(), lse.data_ptr(), rows, vocab,
                                     vocab, None if dl is None else dl.data_ptr(), 0.5,
                                     dz.data_ptr(), s))
    torch.cuda.synchronize()
    return loss.cpu().numpy(), host_bf16(dz)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: "r{}_v{}".format(*c[:2]))
def test_cross_entropy_forward_and_vjp(cuda, oracle, case):
    rows, vocab, std = case
    rng = np.random.default_rng(3)
    z, t = _inputs(oracle, rng, rows, vocab, std)
    dloss = rng.standard_normal(rows).astype(np.float32)
    loss, dz = _run(cuda, z, t, dloss)
    zf = oracle.f32_from_bf16(z)
    want = oracle.cross_entropy(zf, t)
    assert np.allclose(loss, want, rtol=1e-5, atol=1e-5), np.max(np.abs(loss - want))
    ref = oracle.cross_entropy_vjp(zf, t, dloss * np.float32(0.5))
    got = oracle.f32_from_bf16(dz)
    bound = 2.0 ** -8 * np.abs(ref) + 1e-6 * np.abs(ref).max(axis=1, keepdims=True)
    assert np.all(np.abs(got - ref) <= bound), np.max(np.abs(got - ref) - bound)


@pytest.mark.gpu
def test_cross_entropy_large_logits_and_inplace(cuda, oracle):
    """Logits far past exp's f32 range (the max is taken out first), and the
    in-place gradient equal bit for bit to the out-of-place one."""
    rng = np.random.default_rng(4)
    z, t = _inputs(oracle, rng, 8, 4096, 1.0)
    zf = oracle.f32_from_bf16(z)
    zf[0] += 300.0
    zf[1] -= 300.0
    zf[2, 7] = 500.0
    z = oracle.bf16_from_f32(zf)
    zf = oracle.f32_from_bf16(z)
    loss, dz = _run(cuda, z, t)
    loss2, dz2 = _run(cuda, z, t, inplace=True)
    assert np.all(np.isfinite(loss))
    want = oracle.cross_entropy(zf, t)
    assert np.allclose(loss, want, rtol=1e-5, atol=1e-4)
    assert np.array_equal(loss, loss2) and np.array_equal(dz, dz2)


@pytest.mark.gpu
def test_cross_entropy_autograd_matches_torch(cuda):
    """The autograd op against PyTorch's f32 cross-entropy, mean over rows."""
    import torch
    import torch.nn.functional as F

    from torobi_b200.glue import cross_entropy

    g = torch.Generator(device=cuda).manual_seed(5)
    z = (torch.randn(3, 50, 2048, device=cuda, generator=g) * 2).bfloat16()
    t = torch.randint(0, 2048, (3, 50), device=cuda, generator=g)
    a = z.clone().requires_grad_(True)
    la = cross_entropy(a, t).mean()
    la.backward()
    la = la.detach()
    b = z.float().clone().requires_grad_(True)
    lb = F.cross_entropy(b.reshape(-1, 2048), t.reshape(-1))
    lb.backward()
    lb = lb.detach()
    assert abs(la.item() - lb.item()) <= 1e-5 * abs(lb.item())
    err = (a.grad.float() - b.grad).abs().max().item()
    assert err <= 2.0 ** -8 * b.grad.abs().max().item()


@pytest.mark.gpu
def test_cross_entropy_errors(cuda):
    import torch

    from torobi_b200._lib import TQ_ERR_INVALID, TQ_ERR_MISALIGNED, lib

    z = torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda)
    t = torch.zeros(4, dtype=torch.int64, device=cuda)
    f = torch.zeros(4, dtype=torch.float32, device=cuda)
    L = lib()
    assert L.tq_cross_entropy_fwd(z.data_ptr(), t.data_ptr(), 4, 64, 32, f.data_ptr(),
                                  f.data_ptr(), None) == TQ_ERR_INVALID
    assert L.tq_cross_entropy_fwd(z.data_ptr(), t.data_ptr(), 4, 0, 64, f.data_ptr(),
                                  f.data_ptr(), None) == TQ_ERR_INVALID
    assert L.tq_cross_entropy_fwd(z.data_ptr() + 1, t.data_ptr(), 4, 64, 64, f.data_ptr(),
                                  f.data_ptr(), None) == TQ_ERR_MISALIGNED
    assert L.tq_cross_entropy_fwd(z.data_ptr(), t.data_ptr(), 0, 64, 64, None, None, None) == 0

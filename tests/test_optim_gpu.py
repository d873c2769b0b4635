"""The fused AdamW / global-norm kernels against the reference's update rule
(engine/src/optimizer.rs:305-352, engine/src/state.rs:353-400), restated in
the oracle."""
from __future__ import annotations

import numpy as np
import pytest


@pytest.mark.gpu
def test_adamw_matches_the_rule_step_by_step(cuda, oracle):
    import torch
    import torobi_b200 as tq

    rng = np.random.default_rng(4)
    n = 100_003  # not a multiple of 4: exercises the scalar tail
    p = rng.standard_normal(n, dtype=np.float32)
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    P, M, V = (torch.from_numpy(a.copy()).to(cuda) for a in (p, m, v))
    Pb = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    for t in range(1, 6):
        g = rng.standard_normal(n, dtype=np.float32)
        G = torch.from_numpy(g).to(cuda)
        p, m, v = oracle.adamw_step(p, g, m, v, t, lr=0.05, weight_decay=0.01)
        tq.adamw_(P, G, M, V, t, lr=0.05, weight_decay=0.01, params_bf16=Pb)
        np.testing.assert_allclose(P.cpu().numpy(), p, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(M.cpu().numpy(), m, rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(V.cpu().numpy(), v, rtol=1e-5, atol=1e-9)
    assert torch.equal(Pb, P.bfloat16())


@pytest.mark.gpu
def test_adamw_first_step_moves_by_lr(cuda):
    """test/optimizer_test.rb:115-127: with bias correction the first AdamW
    step moves each parameter by almost exactly lr, whatever the gradient."""
    import torch
    import torobi_b200 as tq

    n = 4096
    P = torch.randn(n, device=cuda)
    before = P.clone()
    G = torch.randn(n, device=cuda) * 10.0
    M = torch.zeros(n, device=cuda)
    V = torch.zeros(n, device=cuda)
    tq.adamw_(P, G, M, V, 1, lr=0.01)
    moved = (before - P).abs()
    assert torch.allclose(moved, torch.full_like(moved, 0.01), rtol=0.01)


@pytest.mark.gpu
def test_nonfinite_norm_skips_and_clip_scales(cuda, oracle):
    import torch
    import torobi_b200 as tq

    n = 1000
    P = torch.randn(n, device=cuda)
    G = torch.randn(n, device=cuda)
    M = torch.zeros(n, device=cuda)
    V = torch.zeros(n, device=cuda)
    ns = torch.zeros(1, device=cuda)
    # A non-finite gradient norm: nothing moves (engine/src/state.rs:360-370).
    Gbad = G.clone()
    Gbad[17] = float("nan")
    tq.sumsq(Gbad, ns)
    p0 = P.clone()
    tq.adamw_(P, Gbad, M, V, 1, lr=0.1, norm_sq=ns)
    assert torch.equal(P, p0) and torch.count_nonzero(M) == 0
    # The norm itself, and clipping by it (engine/src/state.rs:373-376).
    tq.sumsq(G, ns)
    norm = oracle.global_norm([G.cpu().numpy()])
    assert abs(float(np.sqrt(ns.item())) - norm) / norm < 1e-5
    clip = norm / 4
    tq.adamw_(P, G, M, V, 1, lr=0.1, norm_sq=ns, clip=clip)
    factor = oracle.clip_factor(norm, clip)
    p_ref, m_ref, _ = oracle.adamw_step(p0.cpu().numpy(), G.cpu().numpy() * np.float32(factor),
                                        np.zeros(n, np.float32), np.zeros(n, np.float32), 1, lr=0.1)
    np.testing.assert_allclose(M.cpu().numpy(), m_ref, rtol=1e-4, atol=1e-7)
    np.testing.assert_allclose(P.cpu().numpy(), p_ref, rtol=1e-5, atol=1e-6)

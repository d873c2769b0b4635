"""The CPU oracle, pinned: the reference's own known answers for this path,
the quantization convention's hand-derivable cases, and the committed golden
fixtures.  No GPU needed."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).parent / "golden"


def test_bf16_of_one_tenth(oracle):
    """docs/plan.md:2599 and test/bf16_test.rb: 0.1 stored as bf16 reads back
    0.100097656."""
    v = oracle.round_bf16(np.float32([0.1]))[0]
    assert abs(float(v) - 0.100097656) < 1e-9


def test_golden_quantize_fixture_reproduces(oracle):
    g = np.load(GOLDEN / "quantize.npz")
    for key in sorted(k for k in g.files if k.startswith("w_")):
        tag = key[2:]
        bits, group = (int(v) for v in tag.split("_"))
        c, s, b = oracle.quantize(g[key], bits, group)
        assert np.array_equal(c, g[f"codes_{tag}"])
        assert np.array_equal(s, g[f"scales_{tag}"])
        assert np.array_equal(b, g[f"biases_{tag}"])
        assert np.array_equal(oracle.dequantize(c, s, b, bits, group), g[f"deq_{tag}"])


def test_golden_qlora_fixture_reproduces(oracle):
    g = np.load(GOLDEN / "qlora.npz")
    M, K, N, r, alpha, bits, group = (int(v) for v in g["meta"])
    f = oracle.f32_from_bf16
    y, _ = oracle.qlora_linear_fwd(f(g["x"]), g["codes"], g["scales"], g["biases"], f(g["lora_a"]),
                                   f(g["lora_b"]), alpha / r, bits, group, bias=f(g["bias"]))
    assert np.array_equal(oracle.bf16_from_f32(y), g["y"])
    dx, da, db = oracle.qlora_linear_bwd(f(g["x"]), f(g["dy"]), g["codes"], g["scales"],
                                         g["biases"], f(g["lora_a"]), f(g["lora_b"]), alpha / r,
                                         bits, group)
    assert np.array_equal(oracle.bf16_from_f32(dx), g["dx"])
    assert np.array_equal(oracle.bf16_from_f32(da), g["da"])
    assert np.array_equal(oracle.bf16_from_f32(db), g["db"])


def _group(oracle, values):
    return oracle.bf16_from_f32(np.asarray(values, np.float32).reshape(1, -1))


def test_quantize_convention_by_hand(oracle):
    """A 4-bit group of 32 holding 0..31 / 31 * 1.5 - 0.5 (min -0.5, max 1.0):
    |max| > |min| so scale is negative and the edge is the max; zero must be
    exactly representable; every value's error is at most half a step."""
    vals = np.linspace(-0.5, 1.0, 32, dtype=np.float32)
    w = _group(oracle, vals)
    c, s32, b32 = oracle.quantize_f32_params(w, 4, 32)
    scale, bias = float(s32[0, 0]), float(b32[0, 0])
    wf = oracle.f32_from_bf16(w)[0]
    # scale = -(1.5/15) = -0.1 before the edge fix; edge = 1.0 (bf16 exact);
    # q0 = rint(1.0 / -0.1) = -10, so scale = 1.0 / -10 and bias = 1.0.
    assert bias == 1.0
    assert scale == np.float32(1.0) / np.float32(-10.0)
    q = oracle.unpack_codes(c, 4)[0]
    assert q.min() >= 0 and q.max() <= 15
    assert q[np.argmax(wf)] == 0                # the edge is code 0
    # zero sits exactly on code 10: bias + 10 * scale == 0
    assert np.float32(bias) + np.float32(10) * np.float32(scale) == 0.0
    recon = np.float32(bias) + q.astype(np.float32) * np.float32(scale)
    inside = wf >= bias + 15 * scale            # values the 16 codes can reach
    assert np.all(np.abs(recon - wf)[inside] <= abs(scale) / 2 + 1e-7)


def test_quantize_side_choice_and_zero_groups(oracle):
    # |min| > |max|: positive scale, edge = min, min is code 0.
    w = _group(oracle, np.linspace(-2.0, 0.5, 64))
    c, s, b = oracle.quantize_f32_params(w, 4, 64)
    assert s[0, 0] > 0 and b[0, 0] == -2.0
    assert oracle.unpack_codes(c, 4)[0][0] == 0
    # All zeros: q0 == 0 so bias stays 0; scale is -eps; every code 0.
    w = _group(oracle, np.zeros(64))
    c, s, b = oracle.quantize_f32_params(w, 8, 64)
    assert b[0, 0] == 0.0 and s[0, 0] == np.float32(-1e-7)
    assert np.all(c == 0)
    # A NaN never becomes min/max and quantizes to code 0.
    vals = np.linspace(-1, 1, 32).astype(np.float32)
    vals[4] = np.nan
    c, s, b = oracle.quantize_f32_params(_group(oracle, vals), 4, 32)
    assert np.isfinite(s[0, 0]) and oracle.unpack_codes(c, 4)[0][4] == 0


def test_packing_is_low_bits_first(oracle):
    q = np.arange(16, dtype=np.uint32).reshape(1, 16) % 16
    packed = oracle.pack_codes(q, 4)
    assert packed[0, 0] == 0x76543210 and packed[0, 1] == 0xFEDCBA98
    assert np.array_equal(oracle.unpack_codes(packed, 4), q)
    q8 = np.array([[1, 2, 3, 4]], np.uint32)
    assert oracle.pack_codes(q8, 8)[0, 0] == 0x04030201


def test_dequantize_rounds_once(oracle):
    """w = RNE(scale*q + bias) rounded once from the exact value.  In each case
    below, rounding the product to bf16 first and then the sum would give the
    second number instead."""
    cases = [  # scale, code, bias, once, twice
        (-1.8671875, 13, 23.0, -1.2734375, -1.25),
        (0.75390625, 14, -11.125, -0.5703125, -0.5625),
        (1.5625, 11, -27.25, -10.0625, -10.0),
        (-1.3984375, 14, -4.96875, -24.5, -24.625),
    ]
    for scale, code, bias, once, twice in cases:
        s = oracle.bf16_from_f32(np.float32([[scale]]))
        b = oracle.bf16_from_f32(np.float32([[bias]]))
        codes = oracle.pack_codes(np.full((1, 32), code, np.uint32), 4)
        out = oracle.f32_from_bf16(oracle.dequantize(codes, s, b, 4, 32))
        assert float(out[0, 0]) == once != twice


def test_qmm_oracles_agree_with_dense_math(oracle, rng):
    w = oracle.normal_bf16(rng, (72, 256), 0.02)
    c, s, b = oracle.quantize(w, 4, 64)
    wd = oracle.f32_from_bf16(oracle.dequantize(c, s, b, 4, 64)).astype(np.float64)
    x = oracle.normal_bf16(rng, (20, 256))
    y = oracle.qmm_fwd(x, c, s, b, 4, 64)
    assert oracle.rel_err(y, oracle.f32_from_bf16(x) @ wd.T) < 1e-6
    dy = oracle.normal_bf16(rng, (20, 72))
    dx = oracle.qmm_dx(dy, c, s, b, 4, 64)
    assert oracle.rel_err(dx, oracle.f32_from_bf16(dy) @ wd) < 1e-6


def test_zero_b_adapter_is_the_base_linear(oracle, rng):
    """test/lora_test.rb:140-148: B starts at zero, so adapted == base."""
    x = oracle.f32_from_bf16(oracle.normal_bf16(rng, (16, 128)))
    w = oracle.normal_bf16(rng, (64, 128), 0.02)
    c, s, b = oracle.quantize(w, 4, 64)
    a = oracle.f32_from_bf16(oracle.normal_bf16(rng, (8, 128), 0.125))
    y, _ = oracle.qlora_linear_fwd(x, c, s, b, a, np.zeros((64, 8), np.float32), 2.0)
    base = oracle.round_bf16(oracle.qmm_fwd(oracle.bf16_from_f32(x), c, s, b))
    assert np.array_equal(y, base)


class _AdamWRule:
    """test/optimizer_test.rb:55-82 (AdamWOracle): the rule written out per
    element in Python floats."""

    def __init__(self, lr, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0):
        self.lr, self.b1, self.b2, self.eps, self.wd = lr, beta1, beta2, eps, weight_decay
        self.t = 0
        self.m = {}
        self.v = {}

    def step(self, params):
        import math

        self.t += 1
        out = {}
        for name, (values, grads) in params.items():
            m = self.m.setdefault(name, [0.0] * len(values))
            v = self.v.setdefault(name, [0.0] * len(values))
            new = []
            for i, (value, g) in enumerate(zip(values, grads)):
                m[i] = self.b1 * m[i] + (1 - self.b1) * g
                v[i] = self.b2 * v[i] + (1 - self.b2) * g * g
                m_hat = m[i] / (1 - self.b1 ** self.t)
                v_hat = v[i] / (1 - self.b2 ** self.t)
                nv = value - self.lr * m_hat / (math.sqrt(v_hat) + self.eps)
                new.append(nv - self.lr * self.wd * value)
            out[name] = new
        return out


def test_adamw_oracle_agrees_with_the_rule_step_by_step(oracle):
    """The reference's test_adamw_agrees_with_the_rule_step_by_step
    (test/optimizer_test.rb:86-113): mse of a 2-in 1-out linear with closed-form
    gradients, five steps at lr 0.05, every parameter within 1e-5."""
    rng = np.random.default_rng(5)
    xs = rng.uniform(-1, 1, (4, 2))
    ys = rng.uniform(-1, 1, 4)
    w, b = [0.5, -0.25], [0.125]
    rule = _AdamWRule(lr=0.05)
    p = np.float32([0.5, -0.25, 0.125])
    m = np.zeros(3, np.float32)
    v = np.zeros(3, np.float32)
    for t in range(1, 6):
        pred = xs @ np.array(w) + b[0]
        dpred = 2.0 * (pred - ys) / len(ys)
        dw = [float(np.sum(dpred * xs[:, 0])), float(np.sum(dpred * xs[:, 1]))]
        db = [float(np.sum(dpred))]
        want = rule.step({"w": (w, dw), "b": (b, db)})
        g = np.float32(dw + db)
        p, m, v = oracle.adamw_step(p, g, m, v, t, lr=0.05)
        w, b = want["w"], want["b"]
        np.testing.assert_allclose(p, np.float32(w + b), atol=1e-5)


def test_adamw_first_step_moves_by_lr(oracle):
    """test/optimizer_test.rb:115-127."""
    g = np.float32([3.0, -0.001, 1e4])
    p, _, _ = oracle.adamw_step(np.zeros(3, np.float32), g, np.zeros(3, np.float32),
                                np.zeros(3, np.float32), 1, lr=0.01)
    np.testing.assert_allclose(np.abs(p), 0.01, rtol=0.01)


def test_decoupled_weight_decay_pulls_toward_zero(oracle):
    """test/optimizer_test.rb:129+: decay moves parameters toward zero and
    never enters the moments."""
    p0 = np.float32([1.0, -1.0])
    g = np.float32([0.0, 0.0])
    z = np.zeros(2, np.float32)
    p_plain, m1, v1 = oracle.adamw_step(p0, g, z, z, 1, lr=0.01)
    p_decay, m2, v2 = oracle.adamw_step(p0, g, z, z, 1, lr=0.01, weight_decay=0.5)
    assert np.all(np.abs(p_decay) < np.abs(p_plain))
    assert np.array_equal(m1, m2) and np.array_equal(v1, v2)


def test_cross_entropy_is_logsumexp_minus_target(oracle, rng):
    z = rng.standard_normal((3, 5, 11)).astype(np.float32) * 5
    t = rng.integers(0, 11, (3, 5))
    ce = oracle.cross_entropy(z, t)
    ref = np.log(np.exp(z.astype(np.float64)).sum(-1)) - np.take_along_axis(z, t[..., None], -1)[..., 0]
    np.testing.assert_allclose(ce, ref, rtol=1e-5, atol=1e-5)


def test_trainable_share_of_qwen_r8_qv(oracle):
    """docs/plan.md:2543, test/lora_test.rb:113-128: rank 8 on q_proj and v_proj
    of Qwen2.5-0.5B is 96 tensors and 540,672 parameters."""
    hidden, kv_dim, layers, r = 896, 128, 24, 8
    per_layer = r * hidden + hidden * r + r * hidden + kv_dim * r
    assert 2 * 2 * layers == 96
    assert per_layer * layers == 540_672


def test_decoder_restatement_vjps_match_torch_autograd():
    """The CPU decoder restatement (the timed CPU baseline) differentiates
    RMSNorm, RoPE, causal GQA attention and SwiGLU as torch autograd does in
    f32, to the bf16 rounding of its outputs."""
    import numpy as np
    import torch

    from oracle import decoder as D

    rng = np.random.default_rng(0)
    T, Hq, Hk, Dh = 12, 4, 2, 16
    f = lambda *s: D.rb(rng.standard_normal(s, dtype=np.float32))  # noqa: E731

    def close(a, b, tol=2e-2):
        a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
        return np.max(np.abs(a - b)) <= tol * max(1e-6, np.max(np.abs(b)))

    x, w, dy = f(T, 64), f(64), f(T, 64)
    y, rstd = D.rms_norm(x, w, 1e-6)
    xt = torch.tensor(x, requires_grad=True)
    yt = xt * torch.rsqrt(xt.pow(2).mean(-1, keepdim=True) + 1e-6) * torch.tensor(w)
    yt.backward(torch.tensor(dy))
    assert close(y, yt.detach().numpy()) and close(D.rms_norm_vjp(x, w, rstd, dy), xt.grad)

    q, k, v, do = f(T, Hq, Dh), f(T, Hk, Dh), f(T, Hk, Dh), f(T, Hq, Dh)
    o, p = D.attention(q, k, v)
    qt, kt, vt = (torch.tensor(a, requires_grad=True) for a in (q, k, v))
    ot = torch.nn.functional.scaled_dot_product_attention(
        qt.transpose(0, 1), kt.transpose(0, 1), vt.transpose(0, 1), is_causal=True,
        enable_gqa=True).transpose(0, 1)
    ot.backward(torch.tensor(do))
    assert close(o, ot.detach().numpy())
    for mine, ref in zip(D.attention_vjp(q, k, v, p, do), (qt.grad, kt.grad, vt.grad)):
        assert close(mine, ref)

    cos, sin = D.rope_tables(T, Dh, 1e4)
    r = D.rope(q, cos, sin)
    assert close(D.rope(r, cos, sin, inverse=True), q)  # a rotation: VJP = inverse

    g, u, da = f(T, 32), f(T, 32), f(T, 32)
    gt, ut = torch.tensor(g, requires_grad=True), torch.tensor(u, requires_grad=True)
    at = torch.nn.functional.silu(gt) * ut
    at.backward(torch.tensor(da))
    dg, du = D.swiglu_vjp(g, u, da)
    assert close(D.swiglu(g, u), at.detach().numpy())
    assert close(dg, gt.grad) and close(du, ut.grad)

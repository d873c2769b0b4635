"""Parity of the quantize / dequantize kernels with the oracle: bit-exact.

Shapes are every linear of a Qwen2.5-0.5B-shaped layer (hidden 896,
intermediate 4864, 14/2 heads of dim 64), weights N(0, 0.02) plus 0.1%
outliers at +-0.5, bits {4, 8} x group {32, 64, 128}: the quantize sweep
the benchmark runs, on seeded synthetic weights.
"""
from __future__ import annotations

import numpy as np
import pytest

from _util import bf16_equal, dev_bf16, first_mismatch, host_bf16, host_u32

QWEN_SHAPES = {
    "q_proj/o_proj": (896, 896),
    "k_proj/v_proj": (128, 896),
    "gate_proj/up_proj": (4864, 896),
    "down_proj": (896, 4864),
}


def _check_quantize(tq, oracle, w, bits, group, device):
    codes, scales, biases = oracle.quantize(w, bits, group)
    tc, ts, tb = tq.quantize(dev_bf16(w, device), group, bits)
    got_c = host_u32(tc)
    assert np.array_equal(got_c, codes), first_mismatch(got_c, codes)
    assert bf16_equal(host_bf16(ts), scales), first_mismatch(host_bf16(ts), scales)
    assert bf16_equal(host_bf16(tb), biases), first_mismatch(host_bf16(tb), biases)
    deq = tq.dequantize(tc, ts, tb, group, bits)
    want = oracle.dequantize(codes, scales, biases, bits, group)
    assert bf16_equal(host_bf16(deq), want), first_mismatch(host_bf16(deq), want)


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_quantize_bit_exact_on_qwen_shapes(cuda, oracle, bits, group):
    import torobi_b200 as tq

    rng = np.random.default_rng(1000 + bits * 10 + group)
    for shape in QWEN_SHAPES.values():
        w = oracle.weights_with_outliers(rng, shape)
        _check_quantize(tq, oracle, w, bits, group, cuda)


def _edge_matrix(oracle, cols):
    f = np.float32
    rows = []
    rows.append(np.zeros(cols, f))                                  # all zero
    rows.append(np.full(cols, 0.75, f))                             # constant positive
    rows.append(np.full(cols, -3.0, f))                             # constant negative
    rows.append(-np.abs(np.linspace(0.1, 2.0, cols, dtype=f)))      # all negative
    rows.append(np.abs(np.linspace(0.1, 2.0, cols, dtype=f)))       # all positive
    rows.append(np.linspace(-1.0, 0.5, cols, dtype=f))              # |min| > |max|
    rows.append(np.linspace(-0.5, 1.0, cols, dtype=f))              # |max| > |min|
    rows.append(np.full(cols, 1e-40, f))                            # subnormal (bf16 denormal)
    r = np.linspace(-1e38, 3e38, cols, dtype=f); rows.append(r)     # near the top of the range
    r = np.linspace(-1.0, 1.0, cols, dtype=f); r[3] = np.nan; rows.append(r)   # a NaN element
    r = np.linspace(-1.0, 1.0, cols, dtype=f); r[5] = np.inf; rows.append(r)   # +inf
    r = np.linspace(-1.0, 1.0, cols, dtype=f); r[7] = -np.inf; rows.append(r)  # -inf
    r = np.zeros(cols, f); r[::2] = -0.0; r[1] = 1e-3; rows.append(r)          # signed zeros
    r = np.linspace(1.0, 1.0001, cols, dtype=f); rows.append(r)     # nearly constant: huge q0
    rows.append(np.full(cols, np.nan, f))                           # all NaN
    r = -np.abs(np.linspace(0.1, 2.0, cols, dtype=f))
    r[::3] = 0.0; r[1::3] = -0.0; rows.append(r)                    # zeros of both signs as max
    r = np.linspace(-1.0, 1.0, cols, dtype=f); r[::4] = np.nan; rows.append(r)  # NaN-riddled
    return oracle.bf16_from_f32(np.stack(rows))


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_quantize_edge_values_bit_exact(cuda, oracle, bits, group):
    import torobi_b200 as tq

    _check_quantize(tq, oracle, _edge_matrix(oracle, 256), bits, group, cuda)


def _half_integer_matrix(oracle, bits, cols, rng):
    """Rows whose quotients (w - bias) / scale sit on or next to half-integers:
    the cases where rounding the quotient to f32 decides the code, which the
    kernel resolves with an IEEE division instead of its reciprocal product."""
    f = np.float32
    n = (1 << bits) - 1
    rows = []
    k = np.arange(cols, dtype=f) % (2 * n + 1) / f(2.0)         # 0, 0.5, ..., n: scale 1
    rows.append(k)
    rows.append(-k)
    for c in rng.uniform(0.01, 3.0, size=14).astype(f):
        r = (np.arange(cols, dtype=f) % n + f(0.5)) * c          # (j + 1/2) * c, bf16-rounded
        r[0], r[1] = f(0.0), f(n) * c                             # pin the group range
        rows.append(r)
    return oracle.bf16_from_f32(np.stack(rows))


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_quantize_half_integer_quotients_bit_exact(cuda, oracle, bits, group):
    import torobi_b200 as tq

    rng = np.random.default_rng(60 + bits + group)
    _check_quantize(tq, oracle, _half_integer_matrix(oracle, bits, 512, rng), bits, group, cuda)


def _wide_range_matrix(oracle, cols, rng):
    """Finite groups across the whole bf16 range: N(0, 1) rows scaled by 2^k
    from subnormal to near the largest finite value (the large ones take the
    kernel's division path), and rows of random finite bf16 bit patterns,
    whose groups mix every exponent."""
    f = np.float32
    rows = [oracle.bf16_from_f32(rng.standard_normal(cols).astype(f) * f(2.0) ** k)
            for k in range(-135, 124, 7)]
    pat = rng.integers(0, 0x10000, size=(16, cols), dtype=np.uint32).astype(np.uint16)
    finite = (pat & 0x7F80) != 0x7F80
    rows.append(np.where(finite, pat, np.uint16(0x3F80)).reshape(16, cols))
    return np.concatenate([np.stack(rows[:-1]), rows[-1]])


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_quantize_wide_range_bit_exact(cuda, oracle, bits, group):
    import torobi_b200 as tq

    rng = np.random.default_rng(90 + bits + group)
    _check_quantize(tq, oracle, _wide_range_matrix(oracle, 1024, rng), bits, group, cuda)


@pytest.mark.gpu
def test_quantize_ragged_and_tiny_shapes(cuda, oracle):
    import torobi_b200 as tq

    rng = np.random.default_rng(7)
    for rows, cols in [(1, 32), (3, 64), (5, 96), (7, 128), (33, 160), (1, 4864)]:
        for bits, group in [(4, 32), (8, 32), (4, 64)]:
            if cols % group:
                continue
            w = oracle.normal_bf16(rng, (rows, cols), 0.02)
            _check_quantize(tq, oracle, w, bits, group, cuda)


@pytest.mark.gpu
def test_golden_quantize_fixture(cuda, oracle):
    import torobi_b200 as tq
    from pathlib import Path

    g = np.load(Path(__file__).parent / "golden" / "quantize.npz")
    for key in sorted(k for k in g.files if k.startswith("w_")):
        tag = key[2:]
        bits, group = (int(v) for v in tag.split("_"))
        tc, ts, tb = tq.quantize(dev_bf16(g[key], cuda), group, bits)
        assert np.array_equal(host_u32(tc), g[f"codes_{tag}"])
        assert bf16_equal(host_bf16(ts), g[f"scales_{tag}"])
        assert bf16_equal(host_bf16(tb), g[f"biases_{tag}"])
        deq = tq.dequantize(tc, ts, tb, group, bits)
        assert bf16_equal(host_bf16(deq), g[f"deq_{tag}"])


@pytest.mark.gpu
def test_quantize_errors_and_empty(cuda):
    import torch
    import torobi_b200 as tq

    w = torch.zeros((4, 96), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="divisible"):
        tq.quantize(w, 64, 4)
    with pytest.raises(ValueError, match="bits"):
        tq.quantize(w, 32, 3)
    with pytest.raises(ValueError, match="group size"):
        tq.quantize(w, 16, 4)
    with pytest.raises(ValueError, match="bfloat16"):
        tq.quantize(w.float(), 32, 4)
    with pytest.raises(ValueError, match="CUDA"):
        tq.quantize(w.cpu(), 32, 4)
    empty = torch.zeros((0, 64), dtype=torch.bfloat16, device=cuda)
    c, s, b = tq.quantize(empty, 64, 4)
    assert c.shape == (0, 8) and s.shape == (0, 1) and b.shape == (0, 1)
    d = tq.dequantize(c, s, b, 64, 4)
    assert d.shape == (0, 64)


@pytest.mark.gpu
@pytest.mark.parametrize("bits,group", [(4, 64), (8, 32), (4, 128)])
def test_batched_quantize_and_dequantize_match_the_oracle(cuda, oracle, bits, group):
    """One launch over matrices of every Qwen2.5-0.5B-shaped linear plus
    ragged, tiny and empty ones, bit-exact to the oracle per matrix; more
    than 256 matrices take several launches with the same results."""
    import torch
    import torobi_b200 as tq

    rng = np.random.default_rng(7)
    shapes = list(QWEN_SHAPES.values()) + [(3, group), (1, 4 * group), (0, group), (37, 2 * group)]
    ws = [oracle.normal_bf16(rng, s, 0.02) for s in shapes]
    ws[2][5, : 2 * group] = oracle.bf16_from_f32(np.full(2 * group, np.nan, np.float32))
    got = tq.quantize_batch([dev_bf16(w, cuda) for w in ws], group, bits)
    deq = tq.dequantize_batch(got, group, bits)
    for i, (w, (c, s_, b_), d) in enumerate(zip(ws, got, deq)):
        codes, scales, biases = oracle.quantize(w, bits, group)
        assert np.array_equal(host_u32(c), codes), (i, first_mismatch(host_u32(c), codes))
        assert bf16_equal(host_bf16(s_), scales) and bf16_equal(host_bf16(b_), biases), i
        assert bf16_equal(host_bf16(d), oracle.dequantize(codes, scales, biases, bits, group)), i
    many = [dev_bf16(oracle.normal_bf16(rng, (2 + i % 5, group), 0.1), cuda) for i in range(300)]
    batched = tq.quantize_batch(many, group, bits)
    for w, (c, s_, b_) in zip(many, batched):
        c1, s1, b1 = tq.quantize(w, group, bits)
        assert torch.equal(c, c1) and torch.equal(s_.view(torch.int16), s1.view(torch.int16))
        assert torch.equal(b_.view(torch.int16), b1.view(torch.int16))
    back = tq.dequantize_batch(batched, group, bits)
    for (c, s_, b_), d in zip(batched, back):
        assert torch.equal(d.view(torch.int16), tq.dequantize(c, s_, b_, group, bits).view(torch.int16))
    assert tq.quantize_batch([], group, bits) == []


@pytest.mark.gpu
def test_batched_quantize_refuses_a_bad_job_before_launching(cuda):
    import ctypes

    import torch
    import torobi_b200 as tq
    from torobi_b200._lib import TQ_ERR_INVALID, TqQuantizeJob, lib

    w = torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda)
    codes = torch.full((4, 8), 7, dtype=torch.uint32, device=cuda)
    sb = torch.zeros(4, 1, dtype=torch.bfloat16, device=cuda)
    jobs = (TqQuantizeJob * 2)(
        TqQuantizeJob(w.data_ptr(), 4, 64, codes.data_ptr(), sb.data_ptr(), sb.data_ptr()),
        TqQuantizeJob(w.data_ptr(), 4, 48, codes.data_ptr(), sb.data_ptr(), sb.data_ptr()))
    assert lib().tq_quantize_batch(jobs, 2, 64, 4, None) == TQ_ERR_INVALID
    assert b"job 1" in lib().tq_last_error()
    torch.cuda.synchronize()
    assert int(codes[0, 0]) == 7  # nothing ran
    with pytest.raises(ValueError):
        tq.quantize_batch([w, w[:, :48]], 64, 4)

"""The quantize kernel's division-free rounding, emulated exactly on the CPU.

The kernel (torobi_b200/csrc/quant.cu, quantize_run) takes each element's code
as min(rint(u * P), P - 1), P = 2^bits, with
    rs = RN(1 / scale), q = RN(d * rs / P), r = RN(d - q * scale * P)  (fma),
    u  = sat(RN(q + r * rs / P))                                        (fma.sat),
where the oracle (and MLX's affine formula) takes clamp(rint(RN(d / scale))).
This restates those four roundings in float32/float64 numpy -- the products
are exact in float64 and the last sum is rounded to float32 through an exact
two-sum -- and checks that the codes agree with the IEEE quotient's over the
groups a bf16 matrix can produce: every bf16 element whose quotient lies in
(-1, P + 1), against scales edge / q0 for every bf16 edge mantissa (both
signs) at 4 bits and 16 sampled ones at 8, with every q0, and against sampled
scales (max - min) / (P - 1) with bias 0 (q0 = 0).  The same restatement over
every bf16 edge mantissa at 8 bits (695 M pairs) found no difference either.
"""
from __future__ import annotations

import numpy as np
import pytest

F32 = np.float32


def _rn32_sum(q: np.ndarray, p: np.ndarray) -> np.ndarray:
    """RN32(q + p) for float32 q and float64 p (p exact), exactly."""
    q64 = q.astype(np.float64)
    s = q64 + p
    bb = s - q64
    e = (q64 - (s - bb)) + (p - bb)                    # q + p == s + e exactly
    r = s.astype(F32)
    lo = np.nextafter(r, F32(-np.inf))
    hi = np.nextafter(r, F32(np.inf))
    r64 = r.astype(np.float64)
    up = (s == (r64 + hi.astype(np.float64)) / 2) & (e > 0)  # s on a float32 midpoint:
    dn = (s == (r64 + lo.astype(np.float64)) / 2) & (e < 0)  # the error decides
    return np.where(up, hi, np.where(dn, lo, r))


def kernel_codes(d: np.ndarray, scale: np.ndarray, bits: int) -> np.ndarray:
    p = F32(2 ** bits)
    rs_p = ((F32(1) / scale).astype(F32) / p).astype(F32)
    scale_p = (scale * p).astype(F32)
    q = (d * rs_p).astype(F32)
    r = (d.astype(np.float64) - q.astype(np.float64) * scale_p.astype(np.float64)).astype(F32)
    u = _rn32_sum(q, r.astype(np.float64) * rs_p.astype(np.float64))
    u = np.where(np.isnan(u), F32(0), np.clip(u, 0, 1))
    return np.minimum(np.rint(u.astype(np.float64) * float(p)), float(p) - 1)


def ieee_codes(d: np.ndarray, scale: np.ndarray, bits: int) -> np.ndarray:
    with np.errstate(all="ignore"):
        y = np.rint((d / scale).astype(F32).astype(np.float64))
    return np.clip(np.where(np.isnan(y), 0, y), 0, 2 ** bits - 1)


def _bf16_values(e_lo: int, e_hi: int) -> np.ndarray:
    """Every bf16 value with a biased exponent in [e_lo, e_hi], both signs."""
    ex = np.arange(e_lo, e_hi + 1, dtype=np.uint32)
    bits = ((ex[:, None] << 7) | np.arange(128, dtype=np.uint32)[None, :]).ravel()
    return (np.concatenate([bits, bits | 0x8000]).astype(np.uint32) << 16).view(F32)


@pytest.mark.parametrize("bits,n_edges", [(4, 256), (8, 16)])
def test_rounding_matches_the_ieee_quotient_for_edge_groups(bits, n_edges):
    rng = np.random.default_rng(bits)
    edges = rng.choice(_bf16_values(120, 120), n_edges, replace=False)  # 256: every one
    vs = np.concatenate([_bf16_values(80, 130), F32([0.0])])
    n = checked = 0
    for edge in edges:
        for q0 in range(1, 2 ** bits):
            for sign in (1, -1):
                scale = F32(edge / F32(sign * q0))
                d = (vs - edge).astype(F32)
                with np.errstate(all="ignore"):
                    y = d / scale
                d = d[(y > -1) & (y < 2 ** bits + 1)]
                s = np.full(d.shape, scale, F32)
                bad = np.nonzero(kernel_codes(d, s, bits) != ieee_codes(d, s, bits))[0]
                assert bad.size == 0, (edge, sign * q0, d[bad[0]])
                checked += d.size
        n += 1
    assert checked > 100_000


@pytest.mark.parametrize("bits", [4, 8])
def test_rounding_matches_the_ieee_quotient_for_zero_bias_groups(bits):
    rng = np.random.default_rng(10 + bits)
    n = 400_000
    vals = _bf16_values(100, 140)
    a, b = rng.choice(vals, n), rng.choice(vals, n)
    scale = np.maximum(((np.maximum(a, b) - np.minimum(a, b)) / F32(2 ** bits - 1)).astype(F32),
                       F32(1e-7))
    scale = np.where(rng.random(n) < 0.5, scale, -scale).astype(F32)
    v = (rng.random(n).astype(F32) * F32(2 ** bits + 1) * scale).astype(F32)
    u = v.view(np.uint32)
    v = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).view(F32)   # to bf16
    bad = np.nonzero(kernel_codes(v, scale, bits) != ieee_codes(v, scale, bits))[0]
    assert bad.size == 0, (v[bad[0]], scale[bad[0]])


def test_the_restatement_sees_a_plain_reciprocal_product_fail():
    """Without the residual step (code = rint(RN(d * rs))) the same scan finds
    differences: the check above is able to fail."""
    vs = np.concatenate([_bf16_values(80, 130), F32([0.0])])
    bad = 0
    for edge in _bf16_values(120, 120)[::16]:
        for q0 in range(1, 16):
            scale = F32(edge / F32(-q0))
            d = (vs - edge).astype(F32)
            with np.errstate(all="ignore"):
                y = d / scale
            d = d[(y > -1) & (y < 17)]
            s = np.full(d.shape, scale, F32)
            rs = (F32(1) / s).astype(F32)
            naive = np.clip(np.rint(np.nan_to_num((d * rs).astype(F32)).astype(np.float64)), 0, 15)
            bad += int((naive != ieee_codes(d, s, 4)).sum())
    assert bad > 0

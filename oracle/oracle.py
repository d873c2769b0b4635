"""CPU oracle for the quantized-weight QLoRA path (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module, and only as the checker.  The product
path (``torobi_b200``) never imports it.

Everything is numpy on the host, with bf16 carried as ``uint16`` bit patterns.
The byte/integer work (quantize, dequantize, packing) and the quantized GEMMs
run in the C restatement ``qlora_oracle.c``; the floating-point compositions
around them (the LoRA branch, its VJP, AdamW, global norm, cross-entropy) are
numpy f32 restatements of the reference's rules, each citing the reference
file it follows.

Pinning: the AdamW, LoRA and bf16-rounding restatements are checked against
the reference's own known answers (its optimizer and LoRA tests); parity
unpinned for quantize / dequantize / quantized_matmul, whose arithmetic lives
in MLX 0.32.2, which neither this machine nor the reference tree holds, and
for which the reference has no golden vectors.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import build as _build

_LIB = None


def _cpu_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return " avx512f" in line
    except OSError:
        pass
    return False


def lib():
    """The compiled C oracle (built on first use if missing)."""
    global _LIB
    if _LIB is None:
        out = _build.build()
        name = "liboracle_avx512.so" if _cpu_has_avx512() else "liboracle.so"
        L = ctypes.CDLL(str(Path(out) / name))
        i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
        L.or_quantize.argtypes = [vp, i64, i64, i32, i32, vp, vp, vp]
        L.or_quantize_f32_params.argtypes = [vp, i64, i64, i32, i32, vp, vp, vp]
        L.or_dequantize.argtypes = [vp, vp, vp, i64, i64, i32, i32, vp]
        L.or_qmm_fwd.argtypes = [vp, vp, vp, vp, i64, i64, i64, i32, i32, vp]
        L.or_qmm_dx.argtypes = [vp, vp, vp, vp, i64, i64, i64, i32, i32, vp]
        L.or_gemm_nt.argtypes = [vp, vp, i64, i64, i64, vp]
        L.or_f32_to_bf16.argtypes = [vp, vp, i64]
        L.or_bf16_to_f32.argtypes = [vp, vp, i64]
        L.or_set_num_threads.argtypes = [i32]
        L.or_num_threads.restype = i32
        for fn in (L.or_quantize, L.or_quantize_f32_params, L.or_dequantize, L.or_qmm_fwd,
                   L.or_qmm_dx, L.or_gemm_nt):
            fn.restype = i32
        _LIB = L
    return _LIB


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def set_threads(n: int) -> None:
    lib().or_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().or_num_threads())


# ------------------------------------------------------------------ bf16 ---

def bf16_from_f32(x) -> np.ndarray:
    """f32 -> bf16 bit patterns, round to nearest even (NaN -> 0x7FC0)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    # u + 0x7FFF + lsb wraps in 32 bits only for NaN patterns, replaced below.
    r = ((u + (np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1)))) >> np.uint32(16))
    r = r.astype(np.uint16)
    r[np.isnan(x)] = 0x7FC0
    return r


def f32_from_bf16(h) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    return (h.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x) -> np.ndarray:
    """f32 values rounded to bf16 and back (what storing in bf16 does)."""
    return f32_from_bf16(bf16_from_f32(x))


# ------------------------------------------------- affine quantization -----

def _check_qargs(bits: int, group: int, cols: int) -> None:
    if bits not in (4, 8):
        raise ValueError(f"bits must be 4 or 8, got {bits}")
    if group not in (32, 64, 128):
        raise ValueError(f"group_size must be 32, 64 or 128, got {group}")
    if cols % group != 0:
        raise ValueError(f"the last dimension ({cols}) must be divisible by group_size ({group})")


def quantize(w_bf16: np.ndarray, bits: int = 4, group: int = 64):
    """MLX affine quantize of a bf16 [rows, cols] matrix along its last axis.

    Returns (codes u32 [rows, cols*bits/32], scales bf16 [rows, cols/group],
    biases bf16 [rows, cols/group]).
    """
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    rows, cols = w.shape
    _check_qargs(bits, group, cols)
    codes = np.zeros((rows, cols * bits // 32), np.uint32)
    scales = np.zeros((rows, cols // group), np.uint16)
    biases = np.zeros((rows, cols // group), np.uint16)
    rc = lib().or_quantize(_p(w), rows, cols, bits, group, _p(codes), _p(scales), _p(biases))
    assert rc == 0
    return codes, scales, biases


def quantize_f32_params(w_bf16: np.ndarray, bits: int = 4, group: int = 64):
    """Like ``quantize`` but returns the f32 scale/bias before bf16 storage."""
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    rows, cols = w.shape
    _check_qargs(bits, group, cols)
    codes = np.zeros((rows, cols * bits // 32), np.uint32)
    scales = np.zeros((rows, cols // group), np.float32)
    biases = np.zeros((rows, cols // group), np.float32)
    rc = lib().or_quantize_f32_params(_p(w), rows, cols, bits, group, _p(codes), _p(scales),
                                      _p(biases))
    assert rc == 0
    return codes, scales, biases


def dequantize(codes, scales, biases, bits: int = 4, group: int = 64) -> np.ndarray:
    """bf16 [rows, cols] with w = RNE_bf16(scale * q + bias)."""
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    biases = np.ascontiguousarray(biases, dtype=np.uint16)
    rows = codes.shape[0]
    cols = codes.shape[1] * 32 // bits
    _check_qargs(bits, group, cols)
    out = np.zeros((rows, cols), np.uint16)
    rc = lib().or_dequantize(_p(codes), _p(scales), _p(biases), rows, cols, bits, group, _p(out))
    assert rc == 0
    return out


def unpack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """u32 packed codes -> one integer code per element (low bits first)."""
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    q = (codes[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    return q.reshape(*codes.shape[:-1], codes.shape[-1] * per)


def pack_codes(q: np.ndarray, bits: int) -> np.ndarray:
    per = 32 // bits
    q = np.ascontiguousarray(q, dtype=np.uint32)
    q = q.reshape(*q.shape[:-1], q.shape[-1] // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    return np.bitwise_or.reduce(q << shifts, axis=-1).astype(np.uint32)


def qmm_fwd(x_bf16, codes, scales, biases, bits=4, group=64) -> np.ndarray:
    """f32 y = x . dequant(W)^T, x bf16 [M, K], W [N, K]."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    biases = np.ascontiguousarray(biases, dtype=np.uint16)
    M, K = x.shape
    N = codes.shape[0]
    assert codes.shape[1] * 32 // bits == K
    y = np.zeros((M, N), np.float32)
    rc = lib().or_qmm_fwd(_p(x), _p(codes), _p(scales), _p(biases), M, N, K, bits, group, _p(y))
    assert rc == 0
    return y


def qmm_dx(dy_bf16, codes, scales, biases, bits=4, group=64) -> np.ndarray:
    """f32 dx = dy . dequant(W), dy bf16 [M, N], W [N, K]."""
    dy = np.ascontiguousarray(dy_bf16, dtype=np.uint16)
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    biases = np.ascontiguousarray(biases, dtype=np.uint16)
    M, N = dy.shape
    K = codes.shape[1] * 32 // bits
    assert codes.shape[0] == N
    dx = np.zeros((M, K), np.float32)
    rc = lib().or_qmm_dx(_p(dy), _p(codes), _p(scales), _p(biases), M, N, K, bits, group, _p(dx))
    assert rc == 0
    return dx


def gemm_nt(a_bf16, b_bf16) -> np.ndarray:
    """f32 c = a . b^T for bf16 a [M, K], b [N, K]."""
    a = np.ascontiguousarray(a_bf16, dtype=np.uint16)
    b = np.ascontiguousarray(b_bf16, dtype=np.uint16)
    M, K = a.shape
    N = b.shape[0]
    c = np.zeros((M, N), np.float32)
    rc = lib().or_gemm_nt(_p(a), _p(b), M, N, K, _p(c))
    assert rc == 0
    return c


# ------------------------------------------------------------ LoRA ---------

def _mm(a, b):
    """f32 matmul of f32 arrays (bf16-valued inputs), f64 accumulation."""
    return (a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32)


def qlora_linear_fwd(x, codes, scales, biases, lora_a, lora_b, scale, bits=4, group=64,
                     bias=None):
    """The adapted linear as the reference graph computes it in bf16.

    lib/torobi/dsl/layers.rb:16-25 (y = x W^T (+ b) + LoRA) and
    lib/torobi/lora.rb:79-85 (LoRA = ((x A^T) B^T) * scale), every op's
    result rounded to bf16 the way a bf16 graph stores it.  Inputs are f32
    arrays holding bf16 values; returns (y, down) as f32 arrays of bf16 values.
    """
    xb = bf16_from_f32(x)
    base = round_bf16(qmm_fwd(xb, codes, scales, biases, bits, group))
    if bias is not None:
        base = round_bf16(base + bias[None, :])
    down = round_bf16(_mm(x, lora_a.T))
    up = round_bf16(_mm(down, lora_b.T))
    lora = round_bf16(up * np.float32(scale))
    return round_bf16(base + lora), down


def qlora_linear_bwd(x, dy, codes, scales, biases, lora_a, lora_b, scale, bits=4, group=64):
    """VJP of ``qlora_linear_fwd`` wrt x, A and B (the base is frozen).

    The rules MLX's autodiff applies to that graph (engine/src/executor.rs:163-191):
    d_up = dy*s; dB = d_up^T down; d_down = d_up B; dA = d_down^T x;
    dx = dy dequant(W) + d_down A.  Each product rounded to bf16.
    """
    down = round_bf16(_mm(x, lora_a.T))
    d_up = round_bf16(dy * np.float32(scale))
    d_b = round_bf16(_mm(d_up.T, down))
    d_down = round_bf16(_mm(d_up, lora_b))
    d_a = round_bf16(_mm(d_down.T, x))
    dx_base = round_bf16(qmm_dx(bf16_from_f32(dy), codes, scales, biases, bits, group))
    dx_lora = round_bf16(_mm(d_down, lora_a))
    return round_bf16(dx_base + dx_lora), d_a, d_b


# ------------------------------------------------------------ AdamW --------

def adamw_step(params, grads, m, v, t, lr, beta1=0.9, beta2=0.999, eps=1e-8,
               weight_decay=0.0):
    """One AdamW update in f32, following engine/src/optimizer.rs:305-352.

    ``t`` is the step count AFTER increment (the reference does ``self.t += 1``
    first, optimizer.rs:297).  Returns new (params, m, v); inputs untouched.
    """
    f = np.float32
    p = np.asarray(params, f)
    g = np.asarray(grads, f)
    bias1 = f(1.0) - f(beta1) ** f(t)
    bias2 = f(1.0) - f(beta2) ** f(t)
    m2 = np.asarray(m, f) * f(beta1) + g * (f(1.0) - f(beta1))
    v2 = np.asarray(v, f) * f(beta2) + (g * g) * (f(1.0) - f(beta2))
    m_hat = m2 / bias1
    v_hat = v2 / bias2
    denom = np.sqrt(v_hat) + f(eps)
    nxt = p - (m_hat / denom) * f(lr)
    if weight_decay != 0.0:
        nxt = nxt - p * f(lr * weight_decay)
    return nxt.astype(f), m2.astype(f), v2.astype(f)


def global_norm(arrays) -> float:
    """L2 norm over every array, in f32 (engine/src/optimizer.rs:64-82)."""
    total = np.float32(0.0)
    for a in arrays:
        a = np.asarray(a, np.float32)
        total = np.float32(total + np.float32(np.sum(a * a, dtype=np.float32)))
    return float(np.sqrt(total))


def clip_factor(norm: float, clip) -> float:
    """engine/src/state.rs:373-376: scale by max/norm when norm > max."""
    if clip is not None and norm > clip:
        return float(np.float32(clip) / np.float32(norm))
    return 1.0


# --------------------------------------------------------- cross-entropy ---

def cross_entropy(logits, targets) -> np.ndarray:
    """Per-position logsumexp(logits) - logits[target], in f32
    (engine/src/interp.rs:440-444)."""
    z = np.asarray(logits, np.float32)
    mx = z.max(axis=-1, keepdims=True)
    lse = (mx[..., 0] + np.log(np.sum(np.exp(z - mx), axis=-1, dtype=np.float32)))
    picked = np.take_along_axis(z, np.asarray(targets)[..., None], axis=-1)[..., 0]
    return (lse - picked).astype(np.float32)


def lora_merge(codes, scales, biases, bits, group, a=None, b=None, scale=1.0) -> np.ndarray:
    """f32 [rows, cols] = dequantize(W) + scale * (b @ a), the sum over the
    rank taken in increasing order with every product and sum rounded to f32
    on its own: the merge an adapted linear's export needs (the reference's
    ``W + scale * BA``, lib/torobi/export.rb:118-127)."""
    deq = f32_from_bf16(dequantize(codes, scales, biases, bits, group))
    if a is None:
        return (deq + np.float32(scale) * np.zeros_like(deq)).astype(np.float32)
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    acc = np.zeros(deq.shape, np.float32)
    for i in range(a.shape[0]):
        acc = acc + b[:, i:i + 1] * a[i:i + 1, :]
    return (deq + np.float32(scale) * acc).astype(np.float32)


def cross_entropy_vjp(logits, targets, dloss) -> np.ndarray:
    """VJP of ``cross_entropy`` wrt the logits, in f32: dloss[r] *
    (softmax(logits[r]) - onehot(targets[r])), the gradient MLX derives for
    logsumexp - take_along_axis (engine/src/interp.rs:440-444)."""
    z = np.asarray(logits, np.float32)
    mx = z.max(axis=-1, keepdims=True)
    e = np.exp(z - mx)
    p = e / np.sum(e, axis=-1, keepdims=True, dtype=np.float32)
    t = np.asarray(targets)
    p[np.arange(z.shape[0]), t] -= np.float32(1.0)
    return (p * np.asarray(dloss, np.float32)[:, None]).astype(np.float32)


# ------------------------------------------------------- seeded inputs -----

def normal_bf16(rng: np.random.Generator, shape, std=1.0) -> np.ndarray:
    """bf16 bit patterns of N(0, std) samples (f32 draw, RNE to bf16)."""
    return bf16_from_f32(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))


def weights_with_outliers(rng: np.random.Generator, shape, std=0.02, frac=0.001,
                          outlier=0.5) -> np.ndarray:
    """N(0, std) plus a fraction of entries set to +-outlier (random sign)."""
    w = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
    n = w.size
    k = int(round(n * frac))
    if k:
        idx = rng.choice(n, size=k, replace=False)
        sign = np.where(rng.random(k) < 0.5, -1.0, 1.0).astype(np.float32)
        w.reshape(-1)[idx] = sign * np.float32(outlier)
    return bf16_from_f32(w)


def rel_err(got, want) -> float:
    """max |got - want| / max |want| (the GEMM tolerance metric)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    denom = float(np.max(np.abs(want))) if want.size else 0.0
    if denom == 0.0:
        return float(np.max(np.abs(got))) if got.size else 0.0
    return float(np.max(np.abs(got - want)) / denom)


"""Parity of quantized_matmul (forward and its VJP wrt x) with the oracle.

Tolerance: max |got - want| / max |want| <= 1e-2 (bf16 operands, f32
accumulation, bf16 output) -- the bar the quantized GEMMs are held to.
"""
from __future__ import annotations

import numpy as np
import pytest

from _util import dev_bf16, dev_u32

TOL = 1e-2

# (m, w_rows, w_cols, bits, group): the single-linear workload first, then
# ragged and tail shapes (m not a multiple of the token tile, w_rows not a
# multiple of 128, w_cols with a half K-step at group 32).
CASES = [
    (512, 4864, 896, 4, 64),
    (1, 128, 64, 4, 64),
    (16, 1024, 512, 4, 64),
    (17, 136, 96, 4, 32),
    (100, 200, 256, 8, 128),
    (300, 264, 384, 8, 32),
    (257, 128, 128, 4, 128),
    (129, 392, 640, 4, 32),
    (640, 256, 1024, 8, 64),
    # scale rows 16-byte aligned (groups per row % 8 == 0): scale tiles by TMA
    (257, 392, 1024, 4, 32),
    (1000, 1032, 2048, 4, 128),
    (33, 264, 4096, 8, 64),
    # small m: split-K over f32 partials in a workspace
    (16, 4096, 4096, 4, 64),
    (100, 2048, 2048, 8, 32),
    # large: CTA pairs (cta_group::2) on 256-row weight tiles.  Forward token
    # tile 128 and dX 256, m ragged; then a last tile whose second CTA lies
    # wholly past the weight's rows; 8-bit both ways; both ways at 256.
    (2000, 2304, 2560, 4, 64),
    (1100, 3080, 1024, 8, 32),
    (2048, 2560, 2048, 8, 64),
    (4096, 4096, 4096, 4, 64),
]


def _setup(oracle, seed, m, n, k, bits, group):
    rng = np.random.default_rng(seed)
    x = oracle.normal_bf16(rng, (m, k))
    w = oracle.normal_bf16(rng, (n, k), 0.02)
    dy = oracle.normal_bf16(rng, (m, n))
    c, s, b = oracle.quantize(w, bits, group)
    return x, dy, c, s, b


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: "m{}_n{}_k{}_b{}_g{}".format(*c))
def test_quantized_matmul_forward(cuda, oracle, case):
    import torobi_b200 as tq

    m, n, k, bits, group = case
    x, _, c, s, b = _setup(oracle, 11, m, n, k, bits, group)
    want = oracle.qmm_fwd(x, c, s, b, bits, group)
    y = tq.quantized_matmul(dev_bf16(x, cuda), dev_u32(c, cuda), dev_bf16(s, cuda),
                            dev_bf16(b, cuda), transpose=True, group_size=group, bits=bits)
    got = y.float().cpu().numpy()
    err = oracle.rel_err(got, want)
    assert err <= TOL, f"max rel err {err:.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: "m{}_n{}_k{}_b{}_g{}".format(*c))
def test_quantized_matmul_backward_dx(cuda, oracle, case):
    import torobi_b200 as tq

    m, n, k, bits, group = case
    _, dy, c, s, b = _setup(oracle, 12, m, n, k, bits, group)
    want = oracle.qmm_dx(dy, c, s, b, bits, group)
    dx = tq.quantized_matmul(dev_bf16(dy, cuda), dev_u32(c, cuda), dev_bf16(s, cuda),
                             dev_bf16(b, cuda), transpose=False, group_size=group, bits=bits)
    got = dx.float().cpu().numpy()
    err = oracle.rel_err(got, want)
    assert err <= TOL, f"max rel err {err:.3e}"


@pytest.mark.gpu
def test_quantized_matmul_matches_dequantized_weight(cuda):
    """quantized_matmul(x, W) equals x . dequantize(W)^T computed in f32 by torch
    on the same dequantized bf16 weight (the dequant inside the GEMM is the
    dequantize kernel's, bit for bit, so only accumulation order differs)."""
    import torch
    import torobi_b200 as tq

    torch.manual_seed(0)
    w = (torch.randn(1024, 2048, device=cuda) * 0.02).bfloat16()
    x = torch.randn(384, 2048, device=cuda).bfloat16()
    c, s, b = tq.quantize(w, 64, 4)
    wd = tq.dequantize(c, s, b, 64, 4).float()
    ref = x.float() @ wd.t()
    y = tq.quantized_matmul(x, c, s, b, True, 64, 4).float()
    assert ((y - ref).abs().max() / ref.abs().max()).item() < 4e-3
    dy = torch.randn(384, 1024, device=cuda).bfloat16()
    ref_dx = dy.float() @ wd
    dx = tq.quantized_matmul(dy, c, s, b, False, 64, 4).float()
    assert ((dx - ref_dx).abs().max() / ref_dx.abs().max()).item() < 4e-3


@pytest.mark.gpu
def test_quantized_matmul_argument_errors(cuda):
    import torch
    import torobi_b200 as tq

    w = torch.zeros((128, 256), dtype=torch.bfloat16, device=cuda)
    c, s, b = tq.quantize(w, 64, 4)
    x = torch.zeros((4, 255), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="last dimension"):
        tq.quantized_matmul(x, c, s, b)
    with pytest.raises(ValueError, match="scales"):
        tq.quantized_matmul(torch.zeros((4, 256), dtype=torch.bfloat16, device=cuda), c, s[:, :2], b)
    y = tq.quantized_matmul(torch.zeros((0, 256), dtype=torch.bfloat16, device=cuda), c, s, b)
    assert y.shape == (0, 128)


@pytest.mark.gpu
def test_split_k_matches_the_unsplit_kernel(cuda):
    """The workspace form equals the plain entry point (which never splits)
    to f32 summation order, and refuses a workspace that is too small."""
    import ctypes

    import torch
    import torobi_b200 as tq
    from torobi_b200._lib import check, lib

    torch.manual_seed(3)
    m, n, k = 48, 2048, 4096  # above the small-token kernel's 32, so the tiles split k
    w = (torch.randn(n, k, device=cuda) * 0.02).bfloat16()
    c, s, b = tq.quantize(w, 64, 4)
    x = torch.randn(m, k, device=cuda).bfloat16()
    nbytes = ctypes.c_size_t(0)
    check(lib().tq_qmm_workspace_bytes(m, n, k, 1, 64, 4, ctypes.byref(nbytes)))
    assert nbytes.value > 0
    st = torch.cuda.current_stream().cuda_stream
    y0 = torch.empty(m, n, device=cuda, dtype=torch.bfloat16)
    check(lib().tq_quantized_matmul(x.data_ptr(), c.data_ptr(), s.data_ptr(), b.data_ptr(), m, n,
                                    k, 1, 64, 4, y0.data_ptr(), st))
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=cuda)
    y1 = torch.empty_like(y0)
    check(lib().tq_quantized_matmul_ws(x.data_ptr(), c.data_ptr(), s.data_ptr(), b.data_ptr(), m,
                                       n, k, 1, 64, 4, y1.data_ptr(), ws.data_ptr(), nbytes.value,
                                       st))
    torch.cuda.synchronize()
    err = ((y1.float() - y0.float()).abs().max() / y0.float().abs().max()).item()
    assert err < 1e-2
    rc = lib().tq_quantized_matmul_ws(x.data_ptr(), c.data_ptr(), s.data_ptr(), b.data_ptr(), m,
                                      n, k, 1, 64, 4, y1.data_ptr(), ws.data_ptr(),
                                      nbytes.value - 16, st)
    assert rc != 0 and b"workspace" in lib().tq_last_error()


# The small-token forward (4-bit, up to 32 tokens, k a multiple of 128):
# weights dequantized in registers for warp-level MMAs, k split over a
# cluster.  Token counts across the 8-token tiles, a row count that leaves a
# partial 128-row block, three chunks of k, every group size, and the
# linear's bias through tq_qlora_matmul with rank 0.
SMALL_CASES = [
    # (m, w_rows, w_cols, group, with_bias)
    (1, 2064, 1024, 64, False),
    (3, 256, 8192, 32, True),
    (8, 1024, 384, 128, False),
    (16, 4096, 4096, 64, True),
    (21, 2064, 2048, 32, False),
    (32, 1024, 14336, 64, True),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", SMALL_CASES, ids=lambda c: "m{}_n{}_k{}_g{}_{}".format(
    *c[:4], "bias" if c[4] else "nobias"))
def test_small_token_forward(cuda, oracle, case):
    import torch

    from torobi_b200._lib import check, lib

    m, n, k, group, with_bias = case
    x, _, c, s, b = _setup(oracle, 31 + m, m, n, k, 4, group)
    rng = np.random.default_rng(m)
    bias = oracle.normal_bf16(rng, (n,), 0.5) if with_bias else None
    dx, dc, ds, db = dev_bf16(x, cuda), dev_u32(c, cuda), dev_bf16(s, cuda), dev_bf16(b, cuda)
    dbias = dev_bf16(bias, cuda) if with_bias else None
    y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
    check(lib().tq_qlora_matmul(dx.data_ptr(), dc.data_ptr(), ds.data_ptr(), db.data_ptr(), m, n,
                                k, 1, group, 4, dbias.data_ptr() if with_bias else None, None,
                                None, 0, 0, y.data_ptr(),
                                torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    want = oracle.qmm_fwd(x, c, s, b, 4, group)
    if with_bias:
        want = want + oracle.f32_from_bf16(bias)[None, :]
    got = y.float().cpu().numpy()
    assert np.isfinite(got).all()
    assert oracle.rel_err(got, want) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(28672, 8192), (65536, 4096)], ids=lambda s: "n{}_k{}".format(*s))
def test_small_token_forward_repeated(cuda, shape):
    """Shapes whose small-token launch wraps its six-stage ring and puts two
    CTAs on an SM, over more than one wave: launched again and again, every
    result must hold (a stage refilled under pending reads once corrupted
    one 16-row slab in most such launches).  Reference: the exactly
    dequantized weight in f32."""
    import torch
    import torobi_b200 as tq

    n, k = shape
    g = torch.Generator(device=cuda)
    g.manual_seed(n + k)
    w = (torch.randn(n, k, device=cuda, generator=g) * 0.02).bfloat16()
    c, s, b = tq.quantize(w, 64, 4)
    wd = tq.dequantize(c, s, b, 64, 4).float()
    del w
    for m in (1, 8):
        for _ in range(8):
            x = torch.randn(m, k, device=cuda, generator=g).bfloat16()
            y = tq.quantized_matmul(x, c, s, b, True, 64, 4).float()
            ref = x.float() @ wd.t()
            err = ((y - ref).abs().max() / ref.abs().max()).item()
            assert err <= TOL, (m, err)


# The quantized_matmul shape sweep: Llama-3-8B projections (4096x4096,
# 1024x4096, 14336x4096, 4096x14336) and Llama-3-70B ones (8192x8192,
# 28672x8192, 8192x28672) as (w_rows, w_cols), 4-bit group 64, weights
# N(0, 0.02), x and dY N(0, 1), at every token count of the sweep.  Above 256
# tokens the oracle is evaluated on a sample of token rows that touches every
# token tile (every 37th row and the last two), which keeps it to seconds;
# the kernel still computes the whole product.  Operands are drawn on the
# device (seeded) and the oracle gets the same bf16 values.
SWEEP_SHAPES = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (8192, 8192),
                (28672, 8192), (8192, 28672)]
SWEEP_MS = [16, 128, 1024, 4096, 16384]
_SWEEP_CACHE: dict = {}


def _sweep_weight(oracle, cuda, n, k):
    """Seeded weight of one sweep shape, quantized by the oracle; cached
    (host and device copies) across the cases of that shape."""
    import torch

    from _util import host_bf16

    key = (n, k)
    if key not in _SWEEP_CACHE:
        _SWEEP_CACHE.clear()  # one shape's operands at a time
        g = torch.Generator(device=cuda)
        g.manual_seed(1000 + n + k)
        w = host_bf16((torch.randn(n, k, device=cuda, generator=g) * 0.02).bfloat16())
        c, s, b = oracle.quantize(w, 4, 64)
        del w
        _SWEEP_CACHE[key] = ((c, s, b), (dev_u32(c, cuda), dev_bf16(s, cuda), dev_bf16(b, cuda)))
    return _SWEEP_CACHE[key]


def _sample_rows(m):
    if m <= 256:
        return np.arange(m)
    return np.array(sorted(set(range(0, m, 37)) | {m - 2, m - 1}))


@pytest.mark.gpu
@pytest.mark.parametrize("direction", ["fwd", "dx"])
@pytest.mark.parametrize("m", SWEEP_MS)
@pytest.mark.parametrize("shape", SWEEP_SHAPES, ids=lambda s: "n{}_k{}".format(*s))
def test_quantized_matmul_projection_sweep(cuda, oracle, shape, m, direction):
    import torch
    import torobi_b200 as tq

    from _util import host_bf16

    n, k = shape
    (c, s, b), (dc, ds, db) = _sweep_weight(oracle, cuda, n, k)
    g = torch.Generator(device=cuda)
    g.manual_seed(7 * m + (1 if direction == "dx" else 0))
    inner, n_out = (k, n) if direction == "fwd" else (n, k)
    x = torch.randn(m, inner, device=cuda, generator=g).bfloat16()
    y = tq.quantized_matmul(x, dc, ds, db, transpose=direction == "fwd", group_size=64, bits=4)
    assert y.shape == (m, n_out)
    rows = _sample_rows(m)
    idx = torch.from_numpy(rows).to(cuda)
    xs = host_bf16(x.index_select(0, idx))
    got = y.index_select(0, idx).float().cpu().numpy()
    del x, y
    if direction == "fwd":
        want = oracle.qmm_fwd(xs, c, s, b, 4, 64)
    else:
        want = oracle.qmm_dx(xs, c, s, b, 4, 64)
    assert np.isfinite(got).all()
    err = oracle.rel_err(got, want)
    assert err <= TOL, f"max rel err {err:.3e} over {len(rows)} sampled rows"


_TS_SCRIPT = r"""
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, sys.argv[1] + "/tests")
from _util import dev_bf16, dev_u32
from oracle import oracle
import torch, torobi_b200 as tq
cuda = torch.device("cuda", 0)
worst = 0.0
for (m, n, k, bits, group) in [(2000, 2304, 2560, 4, 64), (4096, 4096, 4096, 4, 64),
                               (1100, 3080, 1024, 8, 32), (700, 1024, 2048, 4, 128)]:
    rng = np.random.default_rng(m + n)
    x = oracle.normal_bf16(rng, (m, k))
    c, s, b = oracle.quantize(oracle.normal_bf16(rng, (n, k), 0.02), bits, group)
    y = tq.quantized_matmul(dev_bf16(x, cuda), dev_u32(c, cuda), dev_bf16(s, cuda),
                            dev_bf16(b, cuda), True, group, bits)
    rows = np.arange(0, m, 7)
    want = oracle.qmm_fwd(np.ascontiguousarray(x[rows]), c, s, b, bits, group)
    worst = max(worst, oracle.rel_err(y.float().cpu().numpy()[rows], want))
print(worst)
"""


@pytest.mark.gpu
def test_tensor_memory_weight_tile_variant(cuda):
    """The forward pair kernel variant whose dequantized weight tile lives in
    tensor memory (opt-in, TQ_QMM_TS=1, read once per process, hence the
    child process) against the oracle, 4- and 8-bit, token tiles 192 and 128
    with ragged edges."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = str(Path(__file__).resolve().parent.parent)
    out = subprocess.run([sys.executable, "-c", _TS_SCRIPT, root], capture_output=True,
                         text=True, timeout=600, env={**os.environ, "TQ_QMM_TS": "1"})
    assert out.returncode == 0, out.stderr[-2000:]
    err = float(out.stdout.strip().splitlines()[-1])
    assert err <= TOL, f"max rel err {err:.3e}"


# tq_qlora_matmul_accumulate: y = RNE(RNE(result) + y) through every epilogue
# -- CTA pairs (TMA reduce-add), the single-CTA kernel's TMA reduce-add and
# direct stores (y not 16-byte aligned), and split-K's reduce kernel -- bit
# for bit what a separate bf16 add of the plain result gives.
ACC_CASES = [
    # (m, w_rows, w_cols, transpose, lora_rank, bias, y_misaligned)
    (2048, 1024, 4096, False, 16, False, False),   # pairs, dX with LoRA (k/v-like)
    (1000, 2304, 2560, True, 8, True, False),      # pairs, forward, bias + LoRA
    (257, 128, 1024, True, 0, False, False),       # single CTA, TMA epilogue
    (257, 392, 1024, False, 16, False, True),      # single CTA, direct stores
    (16, 4096, 4096, False, 0, False, False),      # split-K (workspace), reduce kernel
    (3, 256, 8192, True, 0, True, False),          # would be the small-token kernel
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", ACC_CASES,
                         ids=lambda c: "m{}_n{}_k{}_t{}_r{}_b{}_u{}".format(*map(int, c)))
def test_accumulate_equals_a_separate_add(cuda, oracle, case):
    import torch
    import torobi_b200 as tq

    m, n, k, transpose, rank, with_bias, misaligned = case
    torch.manual_seed(7)
    w = (torch.randn(n, k, device=cuda) * 0.02).bfloat16()
    c, s, b = tq.quantize(w, 64, 4)
    k_in, n_out = (k, n) if transpose else (n, k)
    x = torch.randn(m, k_in, device=cuda).bfloat16()
    kw = {}
    if rank:
        kw["lora_up"] = (torch.randn(*((n, rank) if transpose else (rank, k)), device=cuda)
                         * 0.05).bfloat16()
        kw["lora_down"] = torch.randn(m, rank, device=cuda).bfloat16()
    if with_bias:
        kw["bias"] = torch.randn(n_out, device=cuda).bfloat16()
    y0 = torch.randn(m, n_out, device=cuda).bfloat16()
    # The result as the accumulating entry point computes it (into zeros: the
    # small-token kernel, which never accumulates, may differ in the last bit).
    plain = tq.qlora_matmul(x, c, s, b, transpose, 64, 4, **kw)
    alone = tq.qlora_matmul(x, c, s, b, transpose, 64, 4,
                            accumulate=torch.zeros_like(plain), **kw)
    assert ((alone.float() - plain.float()).abs().max()
            / plain.float().abs().max()).item() <= TOL
    want = y0.clone().add_(alone)
    if misaligned:
        buf = torch.empty(m * n_out + 1, dtype=torch.bfloat16, device=cuda)
        acc = buf[1:].view(m, n_out)
        assert acc.data_ptr() % 16 != 0
    else:
        acc = torch.empty_like(y0)
    acc.copy_(y0)
    got = tq.qlora_matmul(x, c, s, b, transpose, 64, 4, accumulate=acc, **kw)
    assert got.data_ptr() == acc.data_ptr()
    torch.cuda.synchronize()
    assert torch.equal(got, want), (got.float() - want.float()).abs().max().item()
    # And against the oracle: the quantized product (no LoRA or bias) plus y0.
    if not rank and not with_bias:
        from _util import host_bf16, host_u32

        fn = oracle.qmm_fwd if transpose else oracle.qmm_dx
        ref = fn(host_bf16(x), host_u32(c), host_bf16(s), host_bf16(b), 4, 64) + \
            y0.float().cpu().numpy()
        assert oracle.rel_err(got.float().cpu().numpy(), ref) <= TOL


@pytest.mark.gpu
def test_accumulate_argument_errors(cuda):
    import torch
    import torobi_b200 as tq

    w = torch.zeros((128, 256), dtype=torch.bfloat16, device=cuda)
    c, s, b = tq.quantize(w, 64, 4)
    x = torch.zeros((4, 256), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="accumulate"):
        tq.qlora_matmul(x, c, s, b, accumulate=torch.zeros((4, 64), dtype=torch.bfloat16,
                                                           device=cuda))
    with pytest.raises(ValueError, match="accumulate"):
        tq.qlora_matmul(x, c, s, b, accumulate=torch.zeros((4, 128), dtype=torch.float32,
                                                           device=cuda))


@pytest.mark.gpu
def test_quantized_matmul_random_shapes(cuda):
    """Seeded random shapes across every plan -- the small-token kernel,
    single CTAs with and without split-K, CTA pairs with ragged token and
    weight tiles, scale rows that are or are not 16-byte aligned -- forward
    and dX, 4- and 8-bit, every group size, plain and accumulating, against
    the exactly dequantized weight in f32."""
    import random

    import torch
    import torobi_b200 as tq

    rnd = random.Random(1202)
    for trial in range(24):
        bits = rnd.choice((4, 8))
        group = rnd.choice((32, 64, 128))
        m = rnd.choice((rnd.randint(1, 40), rnd.randint(41, 700), rnd.randint(701, 3000)))
        n = 8 * rnd.randint(1, 512)
        k = group * rnd.randint(1, max(1, 4096 // group))
        transpose = rnd.random() < 0.5
        g = torch.Generator(device=cuda)
        g.manual_seed(trial)
        w = (torch.randn(n, k, device=cuda, generator=g) * 0.02).bfloat16()
        c, s, b = tq.quantize(w, group, bits)
        wd = tq.dequantize(c, s, b, group, bits).float()
        k_in = k if transpose else n
        x = torch.randn(m, k_in, device=cuda, generator=g).bfloat16()
        ref = x.float() @ (wd.t() if transpose else wd)
        y = tq.quantized_matmul(x, c, s, b, transpose, group, bits)
        case = (m, n, k, bits, group, transpose)
        assert torch.isfinite(y.float()).all(), case
        err = ((y.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-6)).item()
        assert err <= TOL, (case, err)
        if trial % 3 == 0:
            # Accumulating into zeros gives the result itself (the small-token
            # kernel, which never accumulates, may differ from it in the last
            # bit); into y0 it gives y0 plus that, as a bf16 add would.
            y0 = torch.randn(y.shape, device=cuda, generator=g).bfloat16()
            base = tq.qlora_matmul(x, c, s, b, transpose, group, bits,
                                   accumulate=torch.zeros_like(y0))
            err = ((base.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-6)).item()
            assert err <= TOL, (case, err)
            acc = tq.qlora_matmul(x, c, s, b, transpose, group, bits, accumulate=y0.clone())
            assert torch.equal(acc, y0.clone().add_(base)), case

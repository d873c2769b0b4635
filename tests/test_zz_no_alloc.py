"""tq_quantized_matmul_noalloc: the split-K GEMM whose f32 partials live in a
fixed array inside the library rather than in a workspace the caller
allocates.  It is for callers that cannot call cudaMalloc while they run (a
runtime with no device allocator of its own, or one whose memory belongs to a
pool this code may not draw from).

Checked through the C ABI, on calls in a row of different shapes (each
call's partials overwrite the previous call's in the shared array; the first
call splits the widest, so partials it leaves behind would be read by a later
call that failed to write its own):
- bit for bit against tq_quantized_matmul_ws, the same plan and kernels with a
  caller-allocated workspace;
- against the oracle within the 1e-2 max-relative-error bar of the other
  quantized GEMM tests.
This file is named so that pytest collects it last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from _util import dev_bf16, dev_u32

TOL = 1e-2
LIMIT = 8 << 20  # TQ_NOALLOC_SCRATCH_BYTES

# (m, w_rows, w_cols, transpose, bits, group): each plans a split on a B200.
CALLS = [
    (200, 2048, 4096, 1, 4, 64),   # forward, the largest scratch of the three
    (16, 1024, 8192, 0, 4, 64),    # the input gradient of a decode-sized batch, k split
    (100, 2048, 2048, 0, 8, 32),   # the input gradient, 8-bit codes
    (200, 2048, 4096, 1, 4, 64),   # the first call again, after the others
]


def _workspace_bytes(L, m, n, k, transpose, bits, group):
    b = ctypes.c_size_t()
    assert L.tq_qmm_workspace_bytes(m, n, k, transpose, group, bits, ctypes.byref(b)) == 0
    return b.value


def _operands(oracle, seed, m, n, k, transpose, bits, group):
    rng = np.random.default_rng(seed)
    x = oracle.normal_bf16(rng, (m, k if transpose else n))
    w = oracle.normal_bf16(rng, (n, k), 0.02)
    c, s, b = oracle.quantize(w, bits, group)
    return x, c, s, b


@pytest.mark.gpu
def test_noalloc_matches_the_workspace_entry_point_and_the_oracle(cuda, oracle):
    import torch

    from torobi_b200._lib import lib

    L = lib()
    stream = torch.cuda.current_stream().cuda_stream
    for i, (m, n, k, tr, bits, group) in enumerate(CALLS):
        need = _workspace_bytes(L, m, n, k, tr, bits, group)
        assert 0 < need <= LIMIT, f"call {i} should split within the fixed array ({need} bytes)"
        hx, hc, hs, hb = _operands(oracle, 40 + i, m, n, k, tr, bits, group)
        x, c, s, b = dev_bf16(hx, cuda), dev_u32(hc, cuda), dev_bf16(hs, cuda), dev_bf16(hb, cuda)
        n_out = n if tr else k
        ws = torch.empty(need, dtype=torch.uint8, device=cuda)
        want = torch.empty(m, n_out, dtype=torch.bfloat16, device=cuda)
        rc = L.tq_quantized_matmul_ws(x.data_ptr(), c.data_ptr(), s.data_ptr(), b.data_ptr(), m, n,
                                      k, tr, group, bits, want.data_ptr(), ws.data_ptr(), need,
                                      stream)
        assert rc == 0, L.tq_last_error().decode()
        got = torch.full((m, n_out), float("nan"), dtype=torch.bfloat16, device=cuda)
        rc = L.tq_quantized_matmul_noalloc(x.data_ptr(), c.data_ptr(), s.data_ptr(), b.data_ptr(),
                                           m, n, k, tr, group, bits, got.data_ptr(), stream)
        assert rc == 0, L.tq_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"call {i}: differs from tq_quantized_matmul_ws"
        ref = (oracle.qmm_fwd(hx, hc, hs, hb, bits, group) if tr
               else oracle.qmm_dx(hx, hc, hs, hb, bits, group))
        err = oracle.rel_err(got.float().cpu().numpy(), ref)
        assert err <= TOL, f"call {i}: max rel err {err:.3e} against the oracle"
    status = ctypes.c_int()
    assert L.tq_device_status(ctypes.byref(status), 1) == 0, L.tq_last_error().decode()


@pytest.mark.gpu
def test_noalloc_refuses_a_split_larger_than_the_array(cuda):
    import torch

    from torobi_b200._lib import TQ_ERR_INVALID, lib

    L = lib()
    m, n, k, tr, bits, group = 256, 1152, 4096, 1, 4, 64
    need = _workspace_bytes(L, m, n, k, tr, bits, group)
    if need <= LIMIT:
        pytest.skip(f"this GPU plans {need} bytes for the shape; nothing to refuse")
    x = torch.zeros(m, k, dtype=torch.bfloat16, device=cuda)
    c = torch.zeros(n, k * bits // 32, dtype=torch.int32, device=cuda)
    s = torch.zeros(n, k // group, dtype=torch.bfloat16, device=cuda)
    y = torch.zeros(m, n, dtype=torch.bfloat16, device=cuda)
    rc = L.tq_quantized_matmul_noalloc(x.data_ptr(), c.data_ptr(), s.data_ptr(), s.data_ptr(), m,
                                       n, k, tr, group, bits, y.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == TQ_ERR_INVALID
    assert "fixed" in L.tq_last_error().decode()

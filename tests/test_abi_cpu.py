"""The C ABI without a GPU: the library loads, exports every symbol the
public header declares, and reports argument errors (checked on the host
before any CUDA call) with a status and a message."""
from __future__ import annotations

import ctypes

import pytest


def test_library_exports_every_header_symbol():
    import torobi_b200 as tq

    L = tq.lib()
    names = tq.header_symbols()
    assert len(names) >= 16
    for name in names:
        assert hasattr(L, name), f"{name} declared in include/torobi_b200.h but not exported"
    from torobi_b200._lib import SIGNATURES

    assert set(SIGNATURES) == set(names), "ctypes signatures out of step with the header"


def test_version_and_empty_error():
    import torobi_b200 as tq

    assert tq.lib().tq_version() >= 100


def test_host_side_argument_errors_need_no_gpu():
    import torobi_b200 as tq
    from torobi_b200._lib import TQ_ERR_INVALID, TQ_ERR_UNSUPPORTED

    L = tq.lib()
    dummy = ctypes.c_void_p(16)
    rc = L.tq_quantize(dummy, 4, 96, 64, 4, dummy, dummy, dummy, None)
    assert rc == TQ_ERR_INVALID
    assert b"divisible" in L.tq_last_error()
    rc = L.tq_quantize(dummy, 4, 64, 64, 3, dummy, dummy, dummy, None)
    assert rc == TQ_ERR_UNSUPPORTED and b"bits" in L.tq_last_error()
    rc = L.tq_quantized_matmul(dummy, dummy, dummy, dummy, 4, 12, 64, 1, 64, 4, dummy, None)
    assert rc == TQ_ERR_INVALID and b"multiple of 8" in L.tq_last_error()
    rc = L.tq_qlora_matmul(dummy, dummy, dummy, dummy, 4, 16, 64, 1, 64, 4, None, dummy, dummy, 0,
                           4, dummy, None)
    assert rc == TQ_ERR_UNSUPPORTED and b"rank" in L.tq_last_error()
    rc = L.tq_qlora_matmul(dummy, dummy, dummy, dummy, 4, 16, 64, 1, 64, 4, None, dummy, dummy, 12,
                           8, dummy, None)
    assert rc == TQ_ERR_INVALID and b"ld_down" in L.tq_last_error()
    rc = L.tq_lora_down(dummy, dummy, 4, 64, 72, 1.0, dummy, None, 0, None)
    assert rc == TQ_ERR_UNSUPPORTED and b"rank" in L.tq_last_error()
    rc = L.tq_adamw(dummy, dummy, dummy, dummy, 10, 0, 0.1, 0.9, 0.999, 1e-8, 0.0, 1.0, None, 0.0,
                    None, None)
    assert rc == TQ_ERR_INVALID and b"step count" in L.tq_last_error()
    rc = L.tq_lora_grad(dummy, dummy, 4, 8, 12, 8, 0, 0, dummy, None)
    assert rc == TQ_ERR_INVALID and b"multiple of 8" in L.tq_last_error()
    rc = L.tq_add_rmsnorm_fwd(dummy, dummy, dummy, 4, 12, 1e-6, dummy, dummy, None, None)
    assert rc == TQ_ERR_INVALID and b"multiple of 8" in L.tq_last_error()
    p = 1 << 20  # 16-byte aligned stand-in addresses; nothing is dereferenced
    rows, hid = 4, 64
    for s_ptr, y_ptr in ((p, p + 4096), (p + (1 << 16), p + 64)):  # s over x; y over x
        rc = L.tq_add_rmsnorm_fwd(p, p + (1 << 14), p + (1 << 15), rows, hid, 1e-6, s_ptr,
                                  y_ptr, None, None)
        assert rc == TQ_ERR_INVALID and b"overlap" in L.tq_last_error()
    rc = L.tq_wait_selftest(10, None)
    assert rc == TQ_ERR_INVALID and b"limit_ns" in L.tq_last_error()
    assert L.tq_dp_comm_abort(None) == 0 and L.tq_dp_comm_destroy(None) == 0


def test_batch_entry_points_check_every_job_first():
    import torobi_b200 as tq
    from torobi_b200._lib import (TQ_ERR_INVALID, TQ_ERR_MISALIGNED, TQ_ERR_UNSUPPORTED,
                                  TqDequantizeJob, TqQuantizeJob)

    L = tq.lib()
    p = 4096  # a 16-byte aligned stand-in address; nothing is dereferenced
    good = TqQuantizeJob(p, 4, 64, p, p, p)
    jobs = (TqQuantizeJob * 3)(good, TqQuantizeJob(p, 0, 64, 0, 0, 0), TqQuantizeJob(p, 4, 96, p, p, p))
    assert L.tq_quantize_batch(jobs, 3, 64, 4, None) == TQ_ERR_INVALID
    assert b"job 2" in L.tq_last_error() and b"divisible" in L.tq_last_error()
    jobs[2] = TqQuantizeJob(p + 8, 4, 64, p, p, p)
    assert L.tq_quantize_batch(jobs, 3, 64, 4, None) == TQ_ERR_MISALIGNED
    assert b"job 2" in L.tq_last_error()
    assert L.tq_quantize_batch(jobs, 3, 48, 4, None) == TQ_ERR_UNSUPPORTED
    assert L.tq_quantize_batch(None, 2, 64, 4, None) == TQ_ERR_INVALID
    djobs = (TqDequantizeJob * 1)(TqDequantizeJob(p, p, p, 4, 64, 0))
    assert L.tq_dequantize_batch(djobs, 1, 64, 4, None) == TQ_ERR_INVALID
    assert b"job 0" in L.tq_last_error() and b"null" in L.tq_last_error()
    assert L.tq_dequantize_batch(djobs, 1, 64, 5, None) == TQ_ERR_UNSUPPORTED


def test_ops_refuse_cpu_tensors():
    import torch
    import torobi_b200 as tq

    w = torch.zeros((8, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        tq.quantize(w, 64, 4)
    with pytest.raises(ValueError, match="CUDA"):
        tq.quantize_batch([w], 64, 4)
    from torobi_b200 import glue

    with pytest.raises(ValueError, match="CUDA"):
        glue.add_rms_norm(w, w, w[0], 1e-6)


def test_attention_argument_errors_need_no_gpu():
    import torobi_b200 as tq
    from torobi_b200._lib import TQ_ERR_INVALID, TQ_ERR_MISALIGNED, TQ_ERR_UNSUPPORTED

    L = tq.lib()
    p = 1 << 20  # 16-byte aligned stand-in address; nothing is dereferenced
    args = lambda heads, kv, dim, scale, out: (p, p, p, 2, 128, heads, kv, dim, scale, 1, out, p, None)
    assert L.tq_attention_fwd(*args(32, 12, 128, 0.1, p)) == TQ_ERR_INVALID
    assert b"multiple of kv_heads" in L.tq_last_error()
    assert L.tq_attention_fwd(*args(32, 8, 96, 0.1, p)) == TQ_ERR_UNSUPPORTED
    assert b"head dim" in L.tq_last_error()
    assert L.tq_attention_fwd(*args(32, 8, 128, 0.0, p)) == TQ_ERR_INVALID
    assert b"scale" in L.tq_last_error()
    assert L.tq_attention_fwd(*args(32, 8, 128, float("nan"), p)) == TQ_ERR_INVALID
    assert L.tq_attention_fwd(*args(32, 8, 128, 0.1, p + 8)) == TQ_ERR_MISALIGNED
    assert L.tq_attention_fwd(*args(32, 8, 128, 0.1, 0)) == TQ_ERR_INVALID
    assert b"null" in L.tq_last_error()
    # Empty batches are valid and touch nothing.
    assert L.tq_attention_fwd(0, 0, 0, 0, 128, 32, 8, 128, 0.1, 1, 0, 0, None) == 0

    need = ctypes.c_size_t(0)
    assert L.tq_attention_bwd_workspace_bytes(2, 129, 4, ctypes.byref(need)) == 0
    assert need.value == 2 * 2 * 4 * 256 * 4  # lse2 and delta, rows padded to 128-row tiles
    assert L.tq_attention_bwd_workspace_bytes(2, 129, 0, ctypes.byref(need)) == TQ_ERR_INVALID

    def bwd(ws_bytes, ws=p):
        return L.tq_attention_bwd(p, p, p, p, p, p, 2, 129, 4, 2, 64, 0.125, 1, p, p, p, ws,
                                  ws_bytes, None)

    assert bwd(need.value - 4) == TQ_ERR_INVALID and b"workspace" in L.tq_last_error()
    assert bwd(need.value, ws=p + 16) == TQ_ERR_MISALIGNED and b"256" in L.tq_last_error()
    assert bwd(need.value, ws=0) == TQ_ERR_INVALID and b"null" in L.tq_last_error()


def test_integration_bindings_match_the_header():
    """The Rust extern block a maintainer would paste binds
    every function of include/torobi_b200.h with the same parameters."""
    import re
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    header = (root / "include" / "torobi_b200.h").read_text()
    decl = {}
    for m in re.finditer(r"^(?:int|const char\*)\s+(tq_\w+)\((.*?)\);", header, flags=re.M | re.S):
        args = [a.strip() for a in m.group(2).split(",") if a.strip() not in ("", "void")]
        decl[m.group(1)] = [a.split()[-1].lstrip("*") for a in args]
    text = (root / "INTEGRATION.md").read_text()
    rust = {}
    for m in re.finditer(r"pub fn (tq_\w+)\((.*?)\)\s*->", text, flags=re.S):
        rust[m.group(1)] = [a.split(":")[0].strip() for a in m.group(2).split(",") if a.strip()]
    assert set(rust) == set(decl), (set(decl) ^ set(rust))
    for name, params in decl.items():
        assert rust[name] == params, name

"""The failure path the kernels share, exercised without a fault: a bounded
device-side wait that nothing satisfies runs out, reports through the device
status word, and leaves the context usable (the kernel ends on its own)."""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

from _util import bf16_equal, dev_bf16, host_bf16


@pytest.mark.gpu
def test_a_lost_wait_reports_a_timeout_and_the_context_stays_usable(cuda, oracle):
    import torch

    import torobi_b200 as tq
    from torobi_b200._lib import TQ_ERR_INVALID, TQ_ERR_TIMEOUT, TqError, lib

    L = lib()
    st = ctypes.c_int(-1)
    assert L.tq_device_status(ctypes.byref(st), 1) in (0, TQ_ERR_TIMEOUT)  # start clean
    assert L.tq_wait_selftest(10, None) == TQ_ERR_INVALID                  # limit refused
    t0 = time.perf_counter()
    assert L.tq_wait_selftest(50_000_000, torch.cuda.current_stream().cuda_stream) == 0
    rc = L.tq_device_status(ctypes.byref(st), 1)                          # syncs the device
    waited = time.perf_counter() - t0
    assert rc == TQ_ERR_TIMEOUT and st.value & 1
    assert 0.04 < waited < 5.0, waited
    assert L.tq_device_status(ctypes.byref(st), 0) == 0 and st.value == 0   # cleared
    with pytest.raises(TqError):                                            # the Python face
        L.tq_wait_selftest(50_000_000, None)
        tq.device_status()
    # The context is fine: a quantize / dequantize round trip still matches.
    rng = np.random.default_rng(3)
    w = oracle.normal_bf16(rng, (64, 256), 0.02)
    c, s, b = tq.quantize(dev_bf16(w, cuda), 64, 4)
    want = oracle.dequantize(*oracle.quantize(w, 4, 64), 4, 64)
    assert bf16_equal(host_bf16(tq.dequantize(c, s, b, 64, 4)), want)
    assert tq.device_status() == 0

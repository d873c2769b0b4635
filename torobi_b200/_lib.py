"""ctypes binding of libtorobi_b200.so (the C ABI declared in include/torobi_b200.h).

There is no fallback: if the library is missing or fails to load, every op
raises.  Build it with ``python -m torobi_b200.build``.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libtorobi_b200.so"
HEADER = _PKG.parent / "include" / "torobi_b200.h"

TQ_OK = 0
TQ_ERR_INVALID = 1
TQ_ERR_UNSUPPORTED = 2
TQ_ERR_MISALIGNED = 3
TQ_ERR_TIMEOUT = 4
TQ_ERR_CUDA = 5
TQ_ERR_NCCL = 6
TQ_DTYPE_F32 = 0
TQ_DTYPE_BF16 = 1

_NAMES = {
    TQ_ERR_INVALID: "invalid argument",
    TQ_ERR_UNSUPPORTED: "unsupported",
    TQ_ERR_MISALIGNED: "misaligned",
    TQ_ERR_TIMEOUT: "device wait timed out",
    TQ_ERR_CUDA: "CUDA error",
    TQ_ERR_NCCL: "NCCL error",
}


class TqError(RuntimeError):
    """A non-zero status from the C ABI, with the library's message."""

    def __init__(self, code: int, message: str):
        self.code = code
        super().__init__(f"[{_NAMES.get(code, code)}] {message}")


_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float

# Argument types of every entry point, in header order.
class TqQuantizeJob(ctypes.Structure):
    """One matrix of tq_quantize_batch (the header's TqQuantizeJob)."""
    _fields_ = [("w", _vp), ("rows", _i64), ("cols", _i64), ("codes", _vp), ("scales", _vp),
                ("biases", _vp)]


class TqDequantizeJob(ctypes.Structure):
    """One matrix of tq_dequantize_batch (the header's TqDequantizeJob)."""
    _fields_ = [("codes", _vp), ("scales", _vp), ("biases", _vp), ("rows", _i64), ("cols", _i64),
                ("w", _vp)]


SIGNATURES = {
    "tq_version": ([], _i32),
    "tq_last_error": ([], ctypes.c_char_p),
    "tq_device_status": ([ctypes.POINTER(_i32), _i32], _i32),
    "tq_wait_selftest": ([_i64, _vp], _i32),
    "tq_quantize_batch": ([ctypes.POINTER(TqQuantizeJob), _i32, _i32, _i32, _vp], _i32),
    "tq_dequantize_batch": ([ctypes.POINTER(TqDequantizeJob), _i32, _i32, _i32, _vp], _i32),
    "tq_quantize": ([_vp, _i64, _i64, _i32, _i32, _vp, _vp, _vp, _vp], _i32),
    "tq_dequantize": ([_vp, _vp, _vp, _i64, _i64, _i32, _i32, _vp, _vp], _i32),
    "tq_quantized_matmul": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _vp, _vp],
                            _i32),
    "tq_qlora_matmul": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _vp, _vp, _vp,
                         _i64, _i64, _vp, _vp], _i32),
    "tq_qmm_workspace_bytes": ([_i64, _i64, _i64, _i32, _i32, _i32, ctypes.POINTER(ctypes.c_size_t)],
                               _i32),
    "tq_quantized_matmul_ws": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _vp, _vp,
                                ctypes.c_size_t, _vp], _i32),
    "tq_qlora_matmul_ws": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _vp, _vp, _vp,
                            _i64, _i64, _vp, _vp, ctypes.c_size_t, _vp], _i32),
    "tq_qlora_matmul_accumulate": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _vp,
                                    _vp, _vp, _i64, _i64, _vp, _vp, ctypes.c_size_t, _vp], _i32),
    "tq_quantized_matmul_noalloc": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _vp,
                                     _vp], _i32),
    "tq_lora_down": ([_vp, _vp, _i64, _i64, _i64, _f32, _vp, _vp, _i64, _vp], _i32),
    "tq_lora_grad": ([_vp, _vp, _i64, _i64, _i64, _i64, _i32, _i32, _vp, _vp], _i32),
    "tq_sumsq": ([_vp, _i64, _vp, _i32, _vp], _i32),
    "tq_adamw": ([_vp, _vp, _vp, _vp, _i64, _i64, _f32, _f32, _f32, _f32, _f32, _f32, _vp, _f32,
                  _vp, _vp], _i32),
    "tq_transpose_to_bf16": ([_vp, _i64, _i64, _vp, _vp], _i32),
    "tq_rmsnorm_fwd": ([_vp, _vp, _i64, _i64, _f32, _vp, _vp, _vp], _i32),
    "tq_add_rmsnorm_fwd": ([_vp, _vp, _vp, _i64, _i64, _f32, _vp, _vp, _vp, _vp], _i32),
    "tq_rmsnorm_bwd": ([_vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp], _i32),
    "tq_attention_fwd": ([_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _vp, _vp, _vp],
                         _i32),
    "tq_attention_bwd_workspace_bytes": ([_i64, _i64, _i64, ctypes.POINTER(ctypes.c_size_t)],
                                         _i32),
    "tq_attention_bwd": ([_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _i32,
                          _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp], _i32),
    "tq_rope": ([_vp, _i64, _i64, _i64, _i64, _vp, _vp, _i32, _vp, _vp], _i32),
    "tq_swiglu_fwd": ([_vp, _vp, _i64, _vp, _vp], _i32),
    "tq_swiglu_bwd": ([_vp, _vp, _vp, _i64, _vp, _vp, _vp], _i32),
    "tq_lora_merge": ([_vp, _vp, _vp, _i64, _i64, _i32, _i32, _vp, _vp, _i64, _f32, _vp, _i32,
                       _vp], _i32),
    "tq_cross_entropy_fwd": ([_vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp], _i32),
    "tq_cross_entropy_bwd": ([_vp, _vp, _vp, _i64, _i64, _i64, _vp, _f32, _vp, _vp], _i32),
    "tq_dp_unique_id": ([_vp], _i32),
    "tq_dp_comm_init": ([ctypes.POINTER(_vp), _vp, _i32, _i32], _i32),
    "tq_dp_allreduce_sum": ([_vp, _vp, _i64, _i32, _vp], _i32),
    "tq_dp_comm_destroy": ([_vp], _i32),
    "tq_dp_comm_abort": ([_vp], _i32),
    "tq_dp_comm_async_error": ([_vp, ctypes.POINTER(_i32)], _i32),
}

_LIB = None


def header_symbols() -> list[str]:
    """Every function the public header declares."""
    text = HEADER.read_text()
    return re.findall(r"^(?:int|const char\*)\s+(tq_\w+)\(", text, flags=re.M)


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built (expected at {LIB_PATH}); "
                "run `python -m torobi_b200.build`")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _LIB = L
    return _LIB


def check(rc: int) -> None:
    if rc != TQ_OK:
        raise TqError(rc, lib().tq_last_error().decode(errors="replace"))


def device_status(clear: bool = True) -> int:
    """Synchronizes and returns the device status word (raises on a timeout)."""
    v = _i32(0)
    check(lib().tq_device_status(ctypes.byref(v), 1 if clear else 0))
    return v.value

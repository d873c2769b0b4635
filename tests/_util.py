"""Host <-> device helpers for the parity tests (bf16 travels as uint16 bits)."""
from __future__ import annotations

import numpy as np


def dev_bf16(a_u16: np.ndarray, device):
    import torch

    a = np.ascontiguousarray(a_u16, dtype=np.uint16)
    return torch.from_numpy(a.view(np.int16)).to(device).view(torch.bfloat16)


def host_bf16(t) -> np.ndarray:
    return t.detach().contiguous().view(__import__("torch").int16).cpu().numpy().view(np.uint16)


def dev_u32(a: np.ndarray, device):
    import torch

    a = np.ascontiguousarray(a, dtype=np.uint32)
    return torch.from_numpy(a.view(np.int32)).to(device).view(torch.uint32)


def host_u32(t) -> np.ndarray:
    import torch

    return t.detach().contiguous().view(torch.int32).cpu().numpy().view(np.uint32)


def host_f32(t) -> np.ndarray:
    import torch

    return t.detach().float().cpu().numpy() if t.dtype != torch.bfloat16 else \
        t.detach().float().cpu().numpy()


def bf16_equal(a: np.ndarray, b: np.ndarray) -> bool:
    """Bitwise equality of bf16 patterns, with every NaN equal to every NaN."""
    a = np.asarray(a, np.uint16)
    b = np.asarray(b, np.uint16)
    if a.shape != b.shape:
        return False
    nan_a = ((a & 0x7F80) == 0x7F80) & ((a & 0x007F) != 0)
    nan_b = ((b & 0x7F80) == 0x7F80) & ((b & 0x007F) != 0)
    return bool(np.all((a == b) | (nan_a & nan_b)))


def first_mismatch(a: np.ndarray, b: np.ndarray) -> str:
    idx = np.argwhere(np.asarray(a) != np.asarray(b))
    if idx.size == 0:
        return "none"
    i = tuple(idx[0])
    return f"{len(idx)} mismatches; first at {i}: got {np.asarray(a)[i]!r} want {np.asarray(b)[i]!r}"

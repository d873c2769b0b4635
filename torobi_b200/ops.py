"""The quantized-weight ops, with MLX's names and argument meaning.

``quantize``, ``dequantize`` and ``quantized_matmul`` take and return torch
CUDA tensors (torch is only the device-memory and stream plumbing here) and
run the hand-written sm_100a kernels of libtorobi_b200.so through its C ABI.
Invalid arguments raise ``ValueError`` before anything is launched, as MLX's
ops do; a failure inside the library raises ``TqError``.

Reference: the engine would reach these through mlx-c (engine/src/mlxc/ops.rs);
the LoRA-adapted linear they serve is lib/torobi/dsl/layers.rb:16-25 with
lib/torobi/lora.rb:79-85.
"""
from __future__ import annotations

import torch

from ._lib import TQ_DTYPE_BF16, TQ_DTYPE_F32, TqDequantizeJob, TqQuantizeJob, check, lib

SUPPORTED_BITS = (4, 8)
SUPPORTED_GROUPS = (32, 64, 128)


class LaunchRecorder:
    """Counts this library's kernel launches and, for the kinds listed in
    ``timed``, brackets each launch with CUDA events on the launching stream
    and accumulates the launch's algorithmic FLOPs and bytes (for the
    roofline)."""

    def __init__(self, timed=("qmm",)):
        self.timed = set(timed)
        self.counts: dict[str, int] = {}
        self.pairs: list[tuple[str, torch.cuda.Event, torch.cuda.Event, float, float]] = []

    def launches(self) -> int:
        return sum(self.counts.values())

    def summary(self) -> dict[str, dict[str, float]]:
        out: dict[str, dict[str, float]] = {}
        for kind, s, e, flops, nbytes in self.pairs:
            d = out.setdefault(kind, {"launches": 0, "ms": 0.0, "flops": 0.0, "bytes": 0.0})
            d["launches"] += 1
            d["ms"] += s.elapsed_time(e)
            d["flops"] += flops
            d["bytes"] += nbytes
        return out


_REC: LaunchRecorder | None = None


def set_recorder(rec: LaunchRecorder | None) -> None:
    global _REC
    _REC = rec


def _launch(kind: str, call, flops: float = 0.0, nbytes: float = 0.0) -> None:
    rec = _REC
    if rec is None:
        check(call())
        return
    rec.counts[kind] = rec.counts.get(kind, 0) + 1
    if kind in rec.timed:
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        check(call())
        e.record()
        rec.pairs.append((kind, s, e, flops, nbytes))
    else:
        check(call())


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need_cuda(op: str, **tensors) -> None:
    for name, t in tensors.items():
        if t is None:
            continue
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"[{op}] {name} must be a torch.Tensor")
        if not t.is_cuda:
            raise ValueError(f"[{op}] {name} must live on a CUDA device (there is no CPU path)")


def _check_bits_group(op: str, group_size: int, bits: int) -> None:
    if bits not in SUPPORTED_BITS:
        raise ValueError(f"[{op}] {bits}-bit quantization is not supported; bits must be 4 or 8")
    if group_size not in SUPPORTED_GROUPS:
        raise ValueError(
            f"[{op}] group size {group_size} is not supported; use 32, 64 or 128")


def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4):
    """Affine-quantize ``w`` along its last axis.

    Returns ``(w_q, scales, biases)``: ``w_q`` uint32 [..., cols*bits/32] with
    codes packed low bits first, ``scales``/``biases`` bf16 [..., cols/group].
    """
    op = "quantize"
    _need_cuda(op, w=w)
    _check_bits_group(op, group_size, bits)
    if w.dim() < 2:
        raise ValueError(f"[{op}] the matrix to quantize needs at least 2 dimensions, got {w.dim()}")
    if w.dtype != torch.bfloat16:
        raise ValueError(f"[{op}] w must be bfloat16, got {w.dtype}")
    cols = w.shape[-1]
    if cols % group_size != 0:
        raise ValueError(
            f"[{op}] the last dimension ({cols}) must be divisible by the group size "
            f"{group_size}; w has shape {tuple(w.shape)}")
    w2 = w.contiguous().reshape(-1, cols)
    rows = w2.shape[0]
    lead = tuple(w.shape[:-1])
    codes = torch.empty(lead + (cols * bits // 32,), dtype=torch.uint32, device=w.device)
    scales = torch.empty(lead + (cols // group_size,), dtype=torch.bfloat16, device=w.device)
    biases = torch.empty_like(scales)
    with torch.cuda.device(w.device):
        _launch("quantize", lambda: lib().tq_quantize(
            _ptr(w2), rows, cols, group_size, bits, _ptr(codes), _ptr(scales), _ptr(biases),
            _stream()))
    return codes, scales, biases


def _check_packed(op: str, w_q, scales, biases, group_size: int, bits: int):
    if w_q.dtype != torch.uint32:
        raise ValueError(f"[{op}] the packed weight must be uint32, got {w_q.dtype}")
    if scales.dtype != torch.bfloat16 or biases.dtype != torch.bfloat16:
        raise ValueError(f"[{op}] scales and biases must be bfloat16")
    cols = w_q.shape[-1] * 32 // bits
    if cols % group_size != 0:
        raise ValueError(f"[{op}] {cols} unpacked columns are not a whole number of groups of "
                         f"{group_size}")
    want = tuple(w_q.shape[:-1]) + (cols // group_size,)
    if tuple(scales.shape) != want or tuple(biases.shape) != want:
        raise ValueError(f"[{op}] scales and biases must have shape {want} for a packed weight "
                         f"of shape {tuple(w_q.shape)}; got {tuple(scales.shape)} and "
                         f"{tuple(biases.shape)}")
    return cols


def dequantize(w_q: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
               group_size: int = 64, bits: int = 4) -> torch.Tensor:
    """bf16 [..., cols] with w = RNE(scale * q + bias)."""
    op = "dequantize"
    _need_cuda(op, w_q=w_q, scales=scales, biases=biases)
    _check_bits_group(op, group_size, bits)
    if w_q.dim() < 2:
        raise ValueError(f"[{op}] the packed matrix needs at least 2 dimensions")
    cols = _check_packed(op, w_q, scales, biases, group_size, bits)
    lead = tuple(w_q.shape[:-1])
    rows = 1
    for d in lead:
        rows *= d
    out = torch.empty(lead + (cols,), dtype=torch.bfloat16, device=w_q.device)
    with torch.cuda.device(w_q.device):
        _launch("dequantize", lambda: lib().tq_dequantize(
            _ptr(w_q.contiguous()), _ptr(scales.contiguous()), _ptr(biases.contiguous()), rows,
            cols, group_size, bits, _ptr(out), _stream()))
    return out


def quantize_batch(ws, group_size: int = 64, bits: int = 4):
    """``quantize`` of every matrix in ``ws`` in one launch (one per 256
    matrices): a list of ``(w_q, scales, biases)`` in the same order."""
    op = "quantize_batch"
    ws = list(ws)
    _check_bits_group(op, group_size, bits)
    outs, keep = [], []
    jobs = (TqQuantizeJob * max(len(ws), 1))()
    for i, w in enumerate(ws):
        _need_cuda(op, w=w)
        if w.dim() < 2 or w.dtype != torch.bfloat16:
            raise ValueError(f"[{op}] matrix {i}: bfloat16 with at least 2 dimensions needed, "
                             f"got {w.dtype} {tuple(w.shape)}")
        cols = w.shape[-1]
        if cols % group_size != 0:
            raise ValueError(f"[{op}] matrix {i}: the last dimension ({cols}) must be divisible "
                             f"by the group size {group_size}")
        if w.device != ws[0].device:
            raise ValueError(f"[{op}] every matrix must be on {ws[0].device}")
        w2 = w.contiguous().reshape(-1, cols)
        lead = tuple(w.shape[:-1])
        codes = torch.empty(lead + (cols * bits // 32,), dtype=torch.uint32, device=w.device)
        scales = torch.empty(lead + (cols // group_size,), dtype=torch.bfloat16, device=w.device)
        biases = torch.empty_like(scales)
        jobs[i] = TqQuantizeJob(_ptr(w2), w2.shape[0], cols, _ptr(codes), _ptr(scales),
                                _ptr(biases))
        keep.append(w2)
        outs.append((codes, scales, biases))
    if ws:
        with torch.cuda.device(ws[0].device):
            _launch("quantize", lambda: lib().tq_quantize_batch(jobs, len(ws), group_size, bits,
                                                                _stream()))
    del keep  # temporaries go back to the caching allocator, reused only in stream order
    return outs


def dequantize_batch(packed, group_size: int = 64, bits: int = 4):
    """``dequantize`` of every ``(w_q, scales, biases)`` in ``packed`` in one
    launch (one per 256): a list of bf16 matrices in the same order."""
    op = "dequantize_batch"
    packed = list(packed)
    _check_bits_group(op, group_size, bits)
    outs, keep = [], []
    jobs = (TqDequantizeJob * max(len(packed), 1))()
    for i, (w_q, scales, biases) in enumerate(packed):
        _need_cuda(op, w_q=w_q, scales=scales, biases=biases)
        if w_q.dim() < 2:
            raise ValueError(f"[{op}] matrix {i}: the packed matrix needs at least 2 dimensions")
        cols = _check_packed(op, w_q, scales, biases, group_size, bits)
        lead = tuple(w_q.shape[:-1])
        rows = 1
        for d in lead:
            rows *= d
        c, s_, b_ = w_q.contiguous(), scales.contiguous(), biases.contiguous()
        out = torch.empty(lead + (cols,), dtype=torch.bfloat16, device=w_q.device)
        jobs[i] = TqDequantizeJob(_ptr(c), _ptr(s_), _ptr(b_), rows, cols, _ptr(out))
        keep += [c, s_, b_]
        outs.append(out)
    if packed:
        with torch.cuda.device(packed[0][0].device):
            _launch("dequantize", lambda: lib().tq_dequantize_batch(jobs, len(packed), group_size,
                                                                    bits, _stream()))
    del keep
    return outs


def lora_merge(w_q: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
               group_size: int = 64, bits: int = 4, lora_a: torch.Tensor | None = None,
               lora_b: torch.Tensor | None = None, scale: float = 1.0,
               dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """[rows, cols] = dequantize(W) + scale * lora_b @ lora_a (f32 sum, each op
    rounded alone), in f32 or bf16: a quantized linear with its LoRA pair
    merged, for export.  lora_a f32 [r, cols], lora_b f32 [rows, r]; neither
    gives the dequantized weight."""
    op = "lora_merge"
    _need_cuda(op, w_q=w_q, scales=scales, biases=biases, lora_a=lora_a, lora_b=lora_b)
    _check_bits_group(op, group_size, bits)
    if w_q.dim() != 2:
        raise ValueError(f"[{op}] the packed weight must be 2-D, got shape {tuple(w_q.shape)}")
    cols = _check_packed(op, w_q, scales, biases, group_size, bits)
    rows = w_q.shape[0]
    if (lora_a is None) != (lora_b is None):
        raise ValueError(f"[{op}] lora_a and lora_b come together")
    rank = 0
    if lora_a is not None:
        if lora_a.dtype != torch.float32 or lora_b.dtype != torch.float32:
            raise ValueError(f"[{op}] the LoRA factors must be float32")
        rank = lora_a.shape[0]
        if tuple(lora_a.shape) != (rank, cols) or tuple(lora_b.shape) != (rows, rank):
            raise ValueError(f"[{op}] lora_a {tuple(lora_a.shape)} and lora_b "
                             f"{tuple(lora_b.shape)} do not fit [{rows}, {cols}]")
        lora_a, lora_b = lora_a.contiguous(), lora_b.contiguous()
    if dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"[{op}] dtype must be float32 or bfloat16")
    out = torch.empty(rows, cols, dtype=dtype, device=w_q.device)
    code = TQ_DTYPE_F32 if dtype == torch.float32 else TQ_DTYPE_BF16
    with torch.cuda.device(w_q.device):
        _launch("lora_merge", lambda: lib().tq_lora_merge(
            _ptr(w_q.contiguous()), _ptr(scales.contiguous()), _ptr(biases.contiguous()), rows,
            cols, group_size, bits, _ptr(lora_a), _ptr(lora_b), rank, float(scale), _ptr(out),
            code, _stream()))
    return out


def _qmm_bytes(m, w_rows, w_cols, transpose, group_size, bits) -> float:
    """Algorithmic bytes of one quantized GEMM: the activation read, the
    packed weight with its scales and biases read, the output written."""
    k_in, n_out = (w_cols, w_rows) if transpose else (w_rows, w_cols)
    return 2.0 * m * k_in + w_rows * w_cols * (bits / 8 + 4 / group_size) + 2.0 * m * n_out


def _gemm_operands(op, x, w_q, scales, biases, transpose, group_size, bits):
    _need_cuda(op, x=x, w_q=w_q, scales=scales, biases=biases)
    _check_bits_group(op, group_size, bits)
    if w_q.dim() != 2:
        raise ValueError(f"[{op}] the packed weight must be 2-D, got shape {tuple(w_q.shape)}")
    if x.dtype != torch.bfloat16:
        raise ValueError(f"[{op}] x must be bfloat16, got {x.dtype}")
    w_cols = _check_packed(op, w_q, scales, biases, group_size, bits)
    w_rows = w_q.shape[0]
    k_in = w_cols if transpose else w_rows
    n_out = w_rows if transpose else w_cols
    if x.shape[-1] != k_in:
        raise ValueError(
            f"[{op}] the last dimension of x ({x.shape[-1]}) does not match the weight: "
            f"expected {k_in} for a [{w_rows}, {w_cols}] weight with transpose={transpose}")
    if w_rows % 8 != 0:
        raise ValueError(f"[{op}] the weight's row count ({w_rows}) must be a multiple of 8")
    x2 = x.contiguous().reshape(-1, k_in)
    return x2, w_rows, w_cols, n_out


def _workspace(m: int, w_rows: int, w_cols: int, transpose: bool, group_size: int, bits: int,
               device) -> tuple[torch.Tensor | None, int]:
    """The split-K workspace a call needs (allocated here, by torch's caching
    allocator; the library itself never allocates)."""
    import ctypes

    nbytes = ctypes.c_size_t(0)
    check(lib().tq_qmm_workspace_bytes(m, w_rows, w_cols, 1 if transpose else 0, group_size,
                                       bits, ctypes.byref(nbytes)))
    if nbytes.value == 0:
        return None, 0
    return torch.empty(nbytes.value, dtype=torch.uint8, device=device), nbytes.value


def quantized_matmul(x: torch.Tensor, w_q: torch.Tensor, scales: torch.Tensor,
                     biases: torch.Tensor, transpose: bool = True, group_size: int = 64,
                     bits: int = 4) -> torch.Tensor:
    """``x . dequant(W)^T`` (transpose) or ``x . dequant(W)``, bf16 out."""
    op = "quantized_matmul"
    x2, w_rows, w_cols, n_out = _gemm_operands(op, x, w_q, scales, biases, transpose,
                                               group_size, bits)
    y = torch.empty(tuple(x.shape[:-1]) + (n_out,), dtype=torch.bfloat16, device=x.device)
    with torch.cuda.device(x.device):
        ws, ws_bytes = _workspace(x2.shape[0], w_rows, w_cols, transpose, group_size, bits,
                                  x.device)
        _launch("qmm", lambda: lib().tq_quantized_matmul_ws(
            _ptr(x2), _ptr(w_q.contiguous()), _ptr(scales.contiguous()), _ptr(biases.contiguous()),
            x2.shape[0], w_rows, w_cols, 1 if transpose else 0, group_size, bits, _ptr(y),
            _ptr(ws), ws_bytes, _stream()), 2.0 * x2.shape[0] * w_rows * w_cols,
            _qmm_bytes(x2.shape[0], w_rows, w_cols, transpose, group_size, bits))
    return y


def qlora_matmul(x: torch.Tensor, w_q: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                 transpose: bool = True, group_size: int = 64, bits: int = 4,
                 bias: torch.Tensor | None = None, lora_up: torch.Tensor | None = None,
                 lora_down: torch.Tensor | None = None,
                 accumulate: torch.Tensor | None = None) -> torch.Tensor:
    """quantized_matmul plus bias and the LoRA up-projection in one kernel.

    transpose: y = x W^T + bias + lora_down . lora_up^T   (lora_up = B [n, r])
    otherwise: y = x W + lora_down . lora_up               (lora_up = A [r, k])
    ``lora_down`` is the [m, r] bf16 down-projection already scaled by alpha/r.
    ``accumulate`` (a contiguous bf16 tensor of y's shape): the result is added
    into it in the GEMM's epilogue, ``accumulate = RNE(RNE(y) + accumulate)``
    (what ``accumulate.add_(y)`` gives), and it is returned.
    """
    op = "qlora_matmul"
    x2, w_rows, w_cols, n_out = _gemm_operands(op, x, w_q, scales, biases, transpose,
                                               group_size, bits)
    _need_cuda(op, bias=bias, lora_up=lora_up, lora_down=lora_down)
    rank = 0
    ld_down = 0
    if lora_up is not None or lora_down is not None:
        if lora_up is None or lora_down is None:
            raise ValueError(f"[{op}] lora_up and lora_down go together")
        rank = lora_down.shape[-1]
        want_up = (w_rows, rank) if transpose else (rank, w_cols)
        if tuple(lora_up.shape) != want_up:
            raise ValueError(f"[{op}] lora_up must have shape {want_up}, got {tuple(lora_up.shape)}")
        if lora_down.reshape(-1, rank).shape[0] != x2.shape[0]:
            raise ValueError(f"[{op}] lora_down must have one row per row of x")
        if lora_up.dtype != torch.bfloat16 or lora_down.dtype != torch.bfloat16:
            raise ValueError(f"[{op}] LoRA operands must be bfloat16")
        if rank not in (8, 16):
            raise ValueError(f"[{op}] LoRA rank must be 8 or 16, got {rank}")
        if lora_down.dim() == 2 and lora_down.stride(1) == 1 and lora_down.stride(0) >= rank:
            # Columns of a stacked down-projection: read in place, row pitch
            # stride(0) (the kernel requires it to be a multiple of 8).
            ld_down = lora_down.stride(0)
            if ld_down % 8 != 0:
                raise ValueError(f"[{op}] lora_down's row pitch ({ld_down}) must be a multiple of 8")
    if bias is not None:
        if not transpose:
            raise ValueError(f"[{op}] a bias is only defined with transpose=True")
        if tuple(bias.shape) != (n_out,) or bias.dtype != torch.bfloat16:
            raise ValueError(f"[{op}] bias must be bfloat16 of shape ({n_out},)")
    shape = tuple(x.shape[:-1]) + (n_out,)
    if accumulate is not None:
        _need_cuda(op, accumulate=accumulate)
        if (tuple(accumulate.shape) != shape or accumulate.dtype != torch.bfloat16
                or not accumulate.is_contiguous() or accumulate.device != x.device):
            raise ValueError(f"[{op}] accumulate must be a contiguous bfloat16 tensor of shape "
                             f"{shape} on {x.device}")
        y = accumulate
        entry = lib().tq_qlora_matmul_accumulate
    else:
        y = torch.empty(shape, dtype=torch.bfloat16, device=x.device)
        entry = lib().tq_qlora_matmul_ws
    up = lora_up.contiguous() if lora_up is not None else None
    if lora_down is None:
        down = None
    elif ld_down:
        down = lora_down
    else:
        down = lora_down.contiguous().reshape(-1, rank)
    b = bias.contiguous() if bias is not None else None
    with torch.cuda.device(x.device):
        ws, ws_bytes = _workspace(x2.shape[0], w_rows, w_cols, transpose, group_size, bits,
                                  x.device)
        _launch("qmm", lambda: entry(
            _ptr(x2), _ptr(w_q.contiguous()), _ptr(scales.contiguous()), _ptr(biases.contiguous()),
            x2.shape[0], w_rows, w_cols, 1 if transpose else 0, group_size, bits, _ptr(b), _ptr(up),
            _ptr(down), ld_down, rank, _ptr(y), _ptr(ws), ws_bytes, _stream()),
            2.0 * x2.shape[0] * w_rows * w_cols,
            _qmm_bytes(x2.shape[0], w_rows, w_cols, transpose, group_size, bits))
    return y


def _lora_rank_ok(rank: int) -> bool:
    return 8 <= rank <= 64 and rank % 8 == 0


def lora_down(x: torch.Tensor, a: torch.Tensor, scale: float, want_transposed: bool = True,
              out_t: torch.Tensor | None = None):
    """Scaled LoRA down-projection on the tensor cores.

    Returns ``(out, out_t)``: ``out`` = RNE(scale * x . a^T) bf16 [m, r] and
    ``out_t`` the same transposed, bf16 [r, ld] with ld = m rounded up to 8
    (columns m.. unused), or None.  ``a`` may stack the A matrices of several
    adapters whose linears share x (r up to 64); ``out_t`` may be given (a
    contiguous [r, ld] bf16 buffer, e.g. rows of a larger stacked one).
    """
    op = "lora_down"
    _need_cuda(op, x=x, a=a, out_t=out_t)
    if x.dtype != torch.bfloat16 or a.dtype != torch.bfloat16:
        raise ValueError(f"[{op}] x and a must be bfloat16")
    rank, k = a.shape
    if not _lora_rank_ok(rank):
        raise ValueError(f"[{op}] LoRA rank must be a multiple of 8 from 8 to 64, got {rank}")
    if x.shape[-1] != k:
        raise ValueError(f"[{op}] x's last dimension ({x.shape[-1]}) must be {k}")
    x2 = x.contiguous().reshape(-1, k)
    m = x2.shape[0]
    out = torch.empty((m, rank), dtype=torch.bfloat16, device=x.device)
    if out_t is not None:
        ld = out_t.shape[-1]
        if (out_t.dtype != torch.bfloat16 or not out_t.is_contiguous() or out_t.dim() != 2
                or out_t.shape[0] != rank or ld < m or ld % 8 != 0):
            raise ValueError(f"[{op}] out_t must be a contiguous bf16 [{rank}, ld] buffer with "
                             f"ld >= {m} a multiple of 8, got {tuple(out_t.shape)}")
    else:
        ld = (m + 7) // 8 * 8
        if want_transposed:
            out_t = torch.empty((rank, ld), dtype=torch.bfloat16, device=x.device)
    with torch.cuda.device(x.device):
        _launch("lora_down", lambda: lib().tq_lora_down(
            _ptr(x2), _ptr(a.contiguous()), m, k, rank, float(scale), _ptr(out), _ptr(out_t), ld,
            _stream()))
    return out, out_t


def lora_grad(x: torch.Tensor, p_t: torch.Tensor, out_layout: int, out: torch.Tensor | None = None,
              accumulate: bool = False) -> torch.Tensor:
    """f32 LoRA weight gradient reduced over the rows of x.

    ``p_t`` is [r, ld] (``lora_down``'s transposed output, ld >= rows of x).
    layout 0 -> [c, r] = x^T p;  layout 1 -> [r, c] = p^T x.
    """
    op = "lora_grad"
    _need_cuda(op, x=x, p_t=p_t, out=out)
    rank, ld = p_t.shape
    if not _lora_rank_ok(rank):
        raise ValueError(f"[{op}] LoRA rank must be a multiple of 8 from 8 to 64, got {rank}")
    c = x.shape[-1]
    x2 = x.contiguous().reshape(-1, c)
    m = x2.shape[0]
    if ld < m or not p_t.is_contiguous():
        raise ValueError(f"[{op}] p_t must be contiguous with at least {m} columns, got {tuple(p_t.shape)}")
    shape = (c, rank) if out_layout == 0 else (rank, c)
    if out is None:
        out = torch.empty(shape, dtype=torch.float32, device=x.device)
        accumulate = False
    elif tuple(out.shape) != shape or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError(f"[{op}] out must be a contiguous float32 tensor of shape {shape}")
    with torch.cuda.device(x.device):
        _launch("lora_grad", lambda: lib().tq_lora_grad(
            _ptr(x2), _ptr(p_t), ld, m, c, rank, out_layout, 1 if accumulate else 0, _ptr(out),
            _stream()))
    return out


def sumsq(x: torch.Tensor, out: torch.Tensor, accumulate: bool = False) -> torch.Tensor:
    _need_cuda("sumsq", x=x, out=out)
    with torch.cuda.device(x.device):
        _launch("sumsq", lambda: lib().tq_sumsq(_ptr(x), x.numel(), _ptr(out),
                                                1 if accumulate else 0, _stream()))
    return out


def adamw_(params: torch.Tensor, grads: torch.Tensor, m: torch.Tensor, v: torch.Tensor, t: int,
           lr: float, beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8,
           weight_decay: float = 0.0, grad_scale: float = 1.0,
           norm_sq: torch.Tensor | None = None, clip: float | None = None,
           params_bf16: torch.Tensor | None = None) -> None:
    """In-place AdamW step over flat f32 buffers (engine/src/optimizer.rs:305-352)."""
    _need_cuda("adamw", params=params, grads=grads, m=m, v=v, norm_sq=norm_sq,
               params_bf16=params_bf16)
    n = params.numel()
    for name, tt in (("grads", grads), ("m", m), ("v", v)):
        if tt.numel() != n or tt.dtype != torch.float32:
            raise ValueError(f"[adamw] {name} must be float32 with {n} elements")
    with torch.cuda.device(params.device):
        _launch("adamw", lambda: lib().tq_adamw(
            _ptr(params), _ptr(grads), _ptr(m), _ptr(v), n, int(t), lr, beta1, beta2, eps,
            weight_decay, grad_scale, _ptr(norm_sq), float(clip) if clip else 0.0,
            _ptr(params_bf16), _stream()))


def transpose_to_bf16(src: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _need_cuda("transpose_to_bf16", src=src, out=out)
    rows, cols = src.shape
    if out is None:
        out = torch.empty((cols, rows), dtype=torch.bfloat16, device=src.device)
    with torch.cuda.device(src.device):
        _launch("transpose", lambda: lib().tq_transpose_to_bf16(
            _ptr(src.contiguous()), rows, cols, _ptr(out), _stream()))
    return out

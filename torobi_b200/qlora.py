"""The adapted linear as a differentiable op, and the flat LoRA parameter store.

``qlora_linear`` is what a model calls for each of its linears: the frozen
base is a quantized weight (codes/scales/biases); an adapter, when present,
adds ``(x A^T) B^T * alpha/rank`` (lib/torobi/lora.rb:79-85) with A
[rank, d_in] and B [d_out, rank] in PyTorch layout (lib/torobi/dsl/layers.rb:18-21).

Forward:  down = lora_down(x, A)            -> [m, r] bf16 (scaled), and its transpose
          y    = qlora_matmul(x, W, bias, B, down)           (one tcgen05 kernel)
Backward: up_g = lora_down(dy, B^T)         -> [m, r] bf16 (scaled), and its transpose
          dx   = qlora_matmul(dy, W, A, up_g, transpose=False)
          dB  += lora_grad(dy, down^T)  ;  dA += lora_grad(x, up_g^T)

Linears that read the same input (a block's q/k/v, its gate/up) run as one
group (``qlora_linears``): their A matrices sit next to each other in the
store, so one down-projection pass over x serves all of them (stacked rank up
to 64), each GEMM reading its adapter's columns in place, and in backward one
pass over x gives every member's dA.

Only the adapter is trainable (lib/torobi/lora.rb:68, :107-111): the base
weight gets no gradient, and the adapter's gradients are accumulated straight
into the store's flat f32 buffer (micro-batch accumulation as in
engine/src/state.rs:418-449), ready for one allreduce and one fused AdamW.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import ops


@dataclass
class QuantizedWeight:
    """A frozen [rows, cols] weight in MLX affine layout."""

    codes: torch.Tensor   # uint32 [rows, cols*bits/32]
    scales: torch.Tensor  # bf16 [rows, cols/group]
    biases: torch.Tensor  # bf16 [rows, cols/group]
    bits: int
    group: int
    bias: torch.Tensor | None = None  # bf16 [rows] (the linear's own bias)

    @property
    def rows(self) -> int:
        return self.codes.shape[0]

    @property
    def cols(self) -> int:
        return self.codes.shape[1] * 32 // self.bits

    @classmethod
    def from_dense(cls, w: torch.Tensor, bits: int = 4, group: int = 64,
                   bias: torch.Tensor | None = None) -> "QuantizedWeight":
        codes, scales, biases = ops.quantize(w, group, bits)
        return cls(codes, scales, biases, bits, group, bias)

    def nbytes(self) -> int:
        n = self.codes.numel() * 4 + self.scales.numel() * 2 + self.biases.numel() * 2
        return n + (self.bias.numel() * 2 if self.bias is not None else 0)


@dataclass
class Adapter:
    """One linear's LoRA pair: views into the store's flat buffers."""

    name: str
    rank: int
    scale: float
    a: torch.Tensor        # f32 [r, d_in]   (master)
    b: torch.Tensor        # f32 [d_out, r]
    a16: torch.Tensor      # bf16 copies the kernels read
    b16: torch.Tensor
    bt16: torch.Tensor     # bf16 [r, d_out] (B transposed, for the backward down-projection)
    ga: torch.Tensor       # f32 gradient views
    gb: torch.Tensor
    group: "AdapterGroup | None" = None
    offset: int = 0        # first row of this adapter's A in the group's stack


@dataclass
class AdapterGroup:
    """Adapters whose linears read the same input, their A matrices stacked
    along the rank in the store's buffers: one down-projection of the input
    for all of them, and one pass for all their dA."""

    name: str
    members: list[Adapter]
    rank: int              # total (sum of the members' ranks)
    scale: float           # alpha / rank, the same for every member
    a16: torch.Tensor      # bf16 [rank, d_in]
    ga: torch.Tensor       # f32 [rank, d_in]


def _round8(n: int) -> int:
    return (n + 7) // 8 * 8


class LoRAStore:
    """Every adapter's parameters, gradients and AdamW moments in flat f32
    buffers, so the data-parallel step is one allreduce and one AdamW launch.

    Offsets are padded to 8 elements so each view (and its bf16 copy) starts on
    a 16-byte boundary, which the TMA copies in the kernels require.
    """

    def __init__(self, device: torch.device):
        self.device = device
        self._specs: list[tuple[str, int, int, int, float, str | None]] = []
        self.adapters: dict[str, Adapter] = {}
        self.groups: dict[str, AdapterGroup] = {}
        self.params = self.grads = self.m = self.v = self.params16 = self.bt16 = None

    def declare(self, name: str, d_in: int, d_out: int, rank: int, alpha: float,
                group: str | None = None) -> None:
        """One adapter; adapters declared with the same ``group`` (linears
        that share an input, same d_in and alpha/rank) are stacked."""
        if self.params is not None:
            raise RuntimeError("the LoRA store is already materialized")
        if rank not in (8, 16):
            raise ValueError(f"LoRA rank must be 8 or 16 on this backend, got {rank}")
        self._specs.append((name, d_in, d_out, rank, float(alpha), group))

    def materialize(self, generator: torch.Generator | None = None) -> None:
        """Allocates the flat buffers; A ~ kaiming_uniform (bound sqrt(6/d_in),
        engine/src/init.rs:42-55), B = 0 (lib/torobi/lora.rb:82).  The A
        matrices of a group are laid out back to back (each rank * d_in, a
        multiple of 8, so no padding falls between them)."""
        by_group: dict[str, list] = {}
        order: list[list] = []
        for spec in self._specs:
            g = spec[5]
            if g is None:
                order.append([spec])
            elif g in by_group:
                by_group[g].append(spec)
            else:
                by_group[g] = [spec]
                order.append(by_group[g])
        for g, members in by_group.items():
            d_ins = {m[1] for m in members}
            scales = {m[4] / m[3] for m in members}
            total = sum(m[3] for m in members)
            if len(d_ins) != 1 or len(scales) != 1 or total > 64:
                raise ValueError(f"adapter group {g}: members need one d_in and one alpha/rank, "
                                 f"and at most 64 stacked ranks")
        total = 0
        offs_a = {}
        for members in order:
            for name, d_in, d_out, rank, alpha, g in members:
                offs_a[name] = total
                total += _round8(rank * d_in)
        t_total = 0
        layout = []
        for name, d_in, d_out, rank, alpha, g in self._specs:
            ob = total
            total += _round8(d_out * rank)
            ot = t_total
            t_total += _round8(rank * d_out)
            layout.append((name, d_in, d_out, rank, alpha, offs_a[name], ob, ot, g))
        dev = self.device
        self.params = torch.zeros(max(total, 8), dtype=torch.float32, device=dev)
        self.grads = torch.zeros_like(self.params)
        self.m = torch.zeros_like(self.params)
        self.v = torch.zeros_like(self.params)
        self.params16 = torch.zeros(max(total, 8), dtype=torch.bfloat16, device=dev)
        self.bt16 = torch.zeros(max(t_total, 8), dtype=torch.bfloat16, device=dev)
        for name, d_in, d_out, rank, alpha, oa, ob, ot, g in layout:
            na, nb = rank * d_in, d_out * rank
            a = self.params[oa:oa + na].view(rank, d_in)
            bound = math.sqrt(6.0 / d_in)
            a.uniform_(-bound, bound, generator=generator)
            self.adapters[name] = Adapter(
                name=name, rank=rank, scale=alpha / rank, a=a,
                b=self.params[ob:ob + nb].view(d_out, rank),
                a16=self.params16[oa:oa + na].view(rank, d_in),
                b16=self.params16[ob:ob + nb].view(d_out, rank),
                bt16=self.bt16[ot:ot + nb].view(rank, d_out),
                ga=self.grads[oa:oa + na].view(rank, d_in),
                gb=self.grads[ob:ob + nb].view(d_out, rank))
        for g, members in by_group.items():
            ads = [self.adapters[m[0]] for m in members]
            d_in = members[0][1]
            o0 = offs_a[members[0][0]]
            r_total = sum(ad.rank for ad in ads)
            grp = AdapterGroup(name=g, members=ads, rank=r_total, scale=ads[0].scale,
                               a16=self.params16[o0:o0 + r_total * d_in].view(r_total, d_in),
                               ga=self.grads[o0:o0 + r_total * d_in].view(r_total, d_in))
            off = 0
            for ad in ads:
                ad.group, ad.offset = grp, off
                off += ad.rank
            self.groups[g] = grp
        self.refresh_bf16(full=True)

    def refresh_bf16(self, full: bool = False) -> None:
        """Re-derives the bf16 copies; the AdamW kernel already wrote params16,
        so after a step only the transposed B copies are rebuilt."""
        if full:
            self.params16.copy_(self.params.to(torch.bfloat16))
        for ad in self.adapters.values():
            ops.transpose_to_bf16(ad.b, out=ad.bt16)

    def numel(self) -> int:
        return sum(ad.a.numel() + ad.b.numel() for ad in self.adapters.values())

    def zero_grad(self) -> None:
        self.grads.zero_()


class _QLoRALinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, trigger, w: QuantizedWeight, ad: Adapter | None):
        # `trigger` is a 0-element tensor that requires grad whenever an
        # adapter is trained, so the backward runs (and accumulates dA, dB)
        # even where x itself needs no gradient (the first layer's input).
        k = x.shape[-1]
        x2 = x.reshape(-1, k)
        if ad is not None:
            down, down_t = ops.lora_down(x2, ad.a16, ad.scale)
            y = ops.qlora_matmul(x2, w.codes, w.scales, w.biases, True, w.group, w.bits,
                                 bias=w.bias, lora_up=ad.b16, lora_down=down)
            ctx.save_for_backward(x2, down_t)
        else:
            y = ops.qlora_matmul(x2, w.codes, w.scales, w.biases, True, w.group, w.bits,
                                 bias=w.bias)
        ctx.w, ctx.ad, ctx.in_shape = w, ad, x.shape
        return y.view(*x.shape[:-1], y.shape[-1])

    @staticmethod
    def backward(ctx, dy):
        w, ad = ctx.w, ctx.ad
        need_dx = ctx.needs_input_grad[0]
        dy2 = dy.reshape(-1, dy.shape[-1])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dx = None
        if ad is not None:
            x2, down_t = ctx.saved_tensors
            up_g, up_g_t = ops.lora_down(dy2, ad.bt16, ad.scale)
            if need_dx:
                dx = ops.qlora_matmul(dy2, w.codes, w.scales, w.biases, False, w.group, w.bits,
                                      lora_up=ad.a16, lora_down=up_g)
            ops.lora_grad(dy2, down_t, 0, out=ad.gb, accumulate=True)
            ops.lora_grad(x2, up_g_t, 1, out=ad.ga, accumulate=True)
        elif need_dx:
            dx = ops.quantized_matmul(dy2, w.codes, w.scales, w.biases, False, w.group, w.bits)
        return (dx.view(ctx.in_shape) if dx is not None else None), None, None, None


class _QLoRAGroup(torch.autograd.Function):
    """Linears reading one input x, the adapted ones' down-projections
    stacked in one pass over x (and their dA in one pass in backward)."""

    @staticmethod
    def forward(ctx, x, trigger, ws, ads, group: AdapterGroup):
        k = x.shape[-1]
        x2 = x.reshape(-1, k)
        down, down_t = ops.lora_down(x2, group.a16, group.scale)
        ys = []
        for w, ad in zip(ws, ads):
            if ad is None:
                y = ops.qlora_matmul(x2, w.codes, w.scales, w.biases, True, w.group, w.bits,
                                     bias=w.bias)
            else:
                y = ops.qlora_matmul(x2, w.codes, w.scales, w.biases, True, w.group, w.bits,
                                     bias=w.bias, lora_up=ad.b16,
                                     lora_down=down[:, ad.offset:ad.offset + ad.rank])
            ys.append(y.view(*x.shape[:-1], y.shape[-1]))
        ctx.save_for_backward(x2, down_t)
        ctx.ws, ctx.ads, ctx.group, ctx.in_shape = ws, ads, group, x.shape
        return tuple(ys)

    @staticmethod
    def backward(ctx, *dys):
        x2, down_t = ctx.saved_tensors
        group = ctx.group
        need_dx = ctx.needs_input_grad[0]
        m = x2.shape[0]
        # Every adapted member's scaled dY.B, transposed, stacked like the A's.
        u_t = torch.empty((group.rank, down_t.shape[1]), dtype=torch.bfloat16, device=x2.device)
        dx = None
        for w, ad, dy in zip(ctx.ws, ctx.ads, dys):
            if dy is None:
                if ad is not None:
                    u_t[ad.offset:ad.offset + ad.rank].zero_()
                continue
            dy2 = dy.reshape(-1, dy.shape[-1])
            if not dy2.is_contiguous():
                dy2 = dy2.contiguous()
            if ad is not None:
                rows = slice(ad.offset, ad.offset + ad.rank)
                up_g, _ = ops.lora_down(dy2, ad.bt16, ad.scale, out_t=u_t[rows])
                ops.lora_grad(dy2, down_t[rows], 0, out=ad.gb, accumulate=True)
                if need_dx:
                    # Members after the first add their dX in the GEMM's epilogue.
                    dx = ops.qlora_matmul(dy2, w.codes, w.scales, w.biases, False, w.group,
                                          w.bits, lora_up=ad.a16, lora_down=up_g, accumulate=dx)
            elif need_dx:
                dx = ops.qlora_matmul(dy2, w.codes, w.scales, w.biases, False, w.group, w.bits,
                                      accumulate=dx)
        ops.lora_grad(x2, u_t, 1, out=group.ga, accumulate=True)
        if dx is not None:
            dx = dx.view(ctx.in_shape)
        elif need_dx:
            dx = torch.zeros(ctx.in_shape, dtype=x2.dtype, device=x2.device)
        return dx, None, None, None, None


_TRIGGERS: dict[torch.device, torch.Tensor] = {}


def _trigger(device: torch.device) -> torch.Tensor:
    t = _TRIGGERS.get(device)
    if t is None:
        t = torch.empty(0, device=device, requires_grad=True)
        _TRIGGERS[device] = t
    return t


def qlora_linear(x: torch.Tensor, w: QuantizedWeight, adapter: Adapter | None = None):
    """y = x W^T (+ bias) (+ LoRA), differentiable wrt x (and the adapter)."""
    trig = _trigger(x.device) if (adapter is not None and torch.is_grad_enabled()) else None
    return _QLoRALinear.apply(x, trig, w, adapter)


def qlora_linears(x: torch.Tensor, ws: list[QuantizedWeight],
                  adapters: list[Adapter | None]) -> tuple[torch.Tensor, ...]:
    """The linears ``ws`` of one input x (with their adapters, or None), as
    ``qlora_linear`` each would give them; when the adapters form one stacked
    group, its down-projection and dA take one pass over x each."""
    groups = {id(ad.group) for ad in adapters if ad is not None}
    grp = next((ad.group for ad in adapters if ad is not None), None)
    if (len(groups) == 1 and grp is not None
            and sorted(id(a) for a in adapters if a is not None) == sorted(map(id, grp.members))):
        trig = _trigger(x.device) if torch.is_grad_enabled() else None
        return _QLoRAGroup.apply(x, trig, list(ws), list(adapters), grp)
    return tuple(qlora_linear(x, w, ad) for w, ad in zip(ws, adapters))

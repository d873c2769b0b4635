"""A Llama-shaped causal LM whose linears run through the quantized-weight path.

The description follows the reference's lib/torobi/models/llama.rb:
pre-norm blocks (``x += attn(norm(x)); x += mlp(norm(x))``, :263-267), GQA
attention with RoPE on q and k and a causal mask (:285-316), SwiGLU
``down((gate * sigmoid(gate)) * up)`` (:320-327), a final RMS norm, and a head
that is the embedding table transposed when tied (:240-259).
RMSNorm is ``x * rsqrt(mean(x^2) + eps) * w`` (engine/src/interp.rs:312-319);
RoPE rotates the first half of each head against the second with angles
``p / theta^(2i/d)`` (engine/src/interp.rs:350-388); the loss is the mean of
``logsumexp(logits) - logits[target]`` in f32 (engine/src/interp.rs:440-444)
over next-token targets.

Every linear of every block is a ``QuantizedWeight`` (MLX affine codes) run by
the tcgen05 quantized GEMM; adapted linears add the fused LoRA branch.  The
norms (each residual add fused into the norm after it), RoPE and SwiGLU
between them are fused kernels (``glue``); attention is this package's
tensor-core kernels (``attention="native"``) or PyTorch's fused SDPA
(``"library"``); the bf16 head is a library GEMM.
The head stays bf16 (a plain library GEMM): QLoRA quantizes the blocks'
linears and keeps the vocabulary projection in the compute dtype.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import glue
from .qlora import Adapter, LoRAStore, QuantizedWeight, qlora_linear, qlora_linears
from .weights import linear_path

LINEARS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")

# Linears of a block that read the same input: their adapters are stacked so
# that one pass over that input serves all of them.
INPUT_GROUPS = {"q_proj": "qkv", "k_proj": "qkv", "v_proj": "qkv", "gate_proj": "gate_up",
                "up_proj": "gate_up"}


def _input_group(layer: int, name: str) -> str | None:
    g = INPUT_GROUPS.get(name)
    return f"layers.{layer}.{g}" if g else None


@dataclass(frozen=True)
class DecoderConfig:
    vocab: int
    hidden: int
    intermediate: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    rope_theta: float
    rms_eps: float
    tie_embeddings: bool
    attention_bias: bool
    bits: int = 4
    group: int = 64
    lora_rank: int = 8
    lora_alpha: float = 16.0
    lora_targets: tuple[str, ...] = ("q_proj", "v_proj")

    def linear_shapes(self) -> dict[str, tuple[int, int]]:
        """[d_out, d_in] of each block linear (PyTorch layout)."""
        h, i = self.hidden, self.intermediate
        q, kv = self.heads * self.head_dim, self.kv_heads * self.head_dim
        return {"q_proj": (q, h), "k_proj": (kv, h), "v_proj": (kv, h), "o_proj": (h, q),
                "gate_proj": (i, h), "up_proj": (i, h), "down_proj": (h, i)}

    def quantized_params(self) -> int:
        return self.layers * sum(o * i for o, i in self.linear_shapes().values())

    def lora_params(self) -> int:
        r = self.lora_rank
        return self.layers * sum(r * (o + i) for n, (o, i) in self.linear_shapes().items()
                                 if n in self.lora_targets)

    def flops_per_token(self, seq: int) -> float:
        """Training FLOPs per token with a frozen base: forward (2P) plus the
        input gradient (2P) through every block linear and the head, plus
        causal attention (forward QK^T and PV, backward twice that)."""
        p = sum(o * i for o, i in self.linear_shapes().values()) * self.layers
        p += self.vocab * self.hidden
        attn_fwd = 2 * 2 * self.heads * self.head_dim * seq / 2 * self.layers
        return 4.0 * p + 3.0 * attn_fwd


# Qwen2.5-0.5B-shaped: hidden 896, intermediate 4864, 24 layers, 14/2 heads of 64,
# tied 151936 vocabulary, q/k/v biases (the qwen2 family), theta 1e6.
QWEN2_5_0_5B = DecoderConfig(vocab=151936, hidden=896, intermediate=4864, layers=24, heads=14,
                             kv_heads=2, head_dim=64, rope_theta=1e6, rms_eps=1e-6,
                             tie_embeddings=True, attention_bias=True, lora_rank=8,
                             lora_alpha=16.0, lora_targets=("q_proj", "v_proj"))

# Llama-3-8B-shaped: hidden 4096, intermediate 14336, 32 layers, 32/8 heads of
# 128, untied 128256 vocabulary, theta 5e5; LoRA r16 alpha 32 on all seven.
LLAMA3_8B = DecoderConfig(vocab=128256, hidden=4096, intermediate=14336, layers=32, heads=32,
                          kv_heads=8, head_dim=128, rope_theta=5e5, rms_eps=1e-5,
                          tie_embeddings=False, attention_bias=False, lora_rank=16,
                          lora_alpha=32.0, lora_targets=LINEARS)

PRESETS = {"qwen2.5-0.5b": QWEN2_5_0_5B, "llama3-8b": LLAMA3_8B}

# Causal GQA attention: this package's tensor-core kernels ("native",
# glue.attention) or PyTorch's fused SDPA ("library").
ATTENTION_IMPLS = ("native", "library")


def tiny_config(**over) -> DecoderConfig:
    """A small model of the same shape family, for tests."""
    base = dict(vocab=1024, hidden=256, intermediate=512, layers=2, heads=4, kv_heads=2,
                head_dim=64, rope_theta=1e4, rms_eps=1e-6, tie_embeddings=True,
                attention_bias=True, lora_rank=8, lora_alpha=16.0,
                lora_targets=("q_proj", "v_proj"))
    base.update(over)
    return DecoderConfig(**base)


def rms_norm_reference(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm composed from PyTorch ops (the tests' f32 restatement)."""
    xf = x.float()
    scale = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * scale * w.float()).to(x.dtype)


def rope_tables(seq: int, dim: int, theta: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    half = dim // 2
    p = torch.arange(seq, dtype=torch.float32, device=device)[:, None]
    i = torch.arange(half, dtype=torch.float32, device=device)[None, :]
    angle = p / torch.pow(torch.tensor(theta, dtype=torch.float32, device=device), 2.0 * i / dim)
    return torch.cos(angle), torch.sin(angle)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """RoPE composed from PyTorch ops, x [B, H, S, D] (the tests' restatement)."""
    half = x.shape[-1] // 2
    xf = x.float()
    a, b = xf[..., :half], xf[..., half:]
    return torch.cat([a * cos - b * sin, b * cos + a * sin], dim=-1).to(x.dtype)


@dataclass
class Block:
    input_norm: torch.Tensor
    post_norm: torch.Tensor
    linears: dict[str, QuantizedWeight] = field(default_factory=dict)
    adapters: dict[str, Adapter | None] = field(default_factory=dict)


class QLoRACausalLM:
    """A causal LM with quantized block linears and a LoRA store: random init,
    or (``source``) a published model's weights quantized as they load."""

    def __init__(self, cfg: DecoderConfig, device: torch.device | str = "cuda", seed: int = 0,
                 dtype: torch.dtype = torch.bfloat16, source=None, attention: str = "library"):
        if attention not in ATTENTION_IMPLS:
            raise ValueError(f"attention must be one of {ATTENTION_IMPLS}, got {attention!r}")
        self.cfg = cfg
        self.attention = attention
        self.device = torch.device(device)
        self.dtype = dtype
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed)
        dev = self.device

        def take(path, shape, init):
            # A published tensor by its path, shape-checked and converted to
            # the compute dtype; or the random initialisation.
            if source is None:
                return init()
            return source.tensor(path, shape, dtype, dev)

        # Embedding table: normal std 0.02 (lib/torobi/dsl/layers.rb:30-35).
        self.embed = take("model.embed_tokens.weight", (cfg.vocab, cfg.hidden),
                          lambda: (torch.randn(cfg.vocab, cfg.hidden, device=dev,
                                               generator=gen) * 0.02).to(dtype))
        self.final_norm = take("model.norm.weight", (cfg.hidden,),
                               lambda: torch.ones(cfg.hidden, dtype=dtype, device=dev))
        if cfg.tie_embeddings:
            self.lm_head = None
        else:
            bound = math.sqrt(6.0 / cfg.hidden)
            self.lm_head = take("lm_head.weight", (cfg.vocab, cfg.hidden),
                                lambda: torch.empty(cfg.vocab, cfg.hidden, device=dev).uniform_(
                                    -bound, bound, generator=gen).to(dtype))
        self.store = LoRAStore(dev)
        shapes = cfg.linear_shapes()
        self.blocks: list[Block] = []
        for li in range(cfg.layers):
            pre = f"model.layers.{li}"
            ones = lambda: torch.ones(cfg.hidden, dtype=dtype, device=dev)  # noqa: E731
            blk = Block(take(f"{pre}.input_layernorm.weight", (cfg.hidden,), ones),
                        take(f"{pre}.post_attention_layernorm.weight", (cfg.hidden,), ones))
            for name, (d_out, d_in) in shapes.items():
                path = linear_path(li, name)
                # Linear weights: kaiming_uniform, bound sqrt(6 / d_in)
                # (engine/src/init.rs:42-55), quantized once at materialisation
                # (at load for a published model).
                bound = math.sqrt(6.0 / d_in)
                w = take(f"{path}.weight", (d_out, d_in),
                         lambda: torch.empty(d_out, d_in, device=dev).uniform_(
                             -bound, bound, generator=gen).to(dtype))
                bias = None
                if cfg.attention_bias and name in ("q_proj", "k_proj", "v_proj"):
                    bias = take(f"{path}.bias", (d_out,),
                                lambda: torch.zeros(d_out, dtype=dtype, device=dev))
                blk.linears[name] = QuantizedWeight.from_dense(w, cfg.bits, cfg.group, bias)
                del w
                if name in cfg.lora_targets:
                    self.store.declare(f"layers.{li}.{name}", d_in, d_out, cfg.lora_rank,
                                       cfg.lora_alpha, group=_input_group(li, name))
            self.blocks.append(blk)
        # The adapter's matrices are fresh whatever the source (they are in
        # no published model): A drawn from the seed, B zero.
        self.store.materialize(gen)
        for li, blk in enumerate(self.blocks):
            for name in shapes:
                blk.adapters[name] = self.store.adapters.get(f"layers.{li}.{name}")
        self._rope_cache: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}

    @classmethod
    def from_pretrained(cls, cfg: DecoderConfig, path, device: torch.device | str = "cuda",
                        seed: int = 0, attention: str = "library") -> "QLoRACausalLM":
        """A published model's safetensors file, every block linear quantized
        on the device as it arrives; the adapter fresh from ``seed``."""
        from .weights import SafetensorsSource

        return cls(cfg, device=device, seed=seed, source=SafetensorsSource(path),
                   attention=attention)

    def _rope(self, seq: int):
        t = self._rope_cache.get(seq)
        if t is None:
            t = rope_tables(seq, self.cfg.head_dim, self.cfg.rope_theta, self.device)
            self._rope_cache[seq] = t
        return t

    def block_forward(self, blk: Block, x: torch.Tensor, h: torch.Tensor,
                      next_norm: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """One pre-norm block on the residual stream ``x`` whose input norm
        ``h`` is already computed; returns the new stream and its norm under
        ``next_norm`` (the next block's input norm, or the final norm).  Each
        residual add is fused with the norm that follows it."""
        cfg = self.cfg
        B, S, H = x.shape
        cos, sin = self._rope(S)
        qkv = ("q_proj", "k_proj", "v_proj")
        q, k, v = qlora_linears(h, [blk.linears[n] for n in qkv], [blk.adapters[n] for n in qkv])
        # [B, S, heads, D] in memory; attention reads the [B, heads, S, D] view.
        q = glue.rope(q.view(B, S, cfg.heads, cfg.head_dim), cos, sin)
        k = glue.rope(k.view(B, S, cfg.kv_heads, cfg.head_dim), cos, sin)
        v = v.view(B, S, cfg.kv_heads, cfg.head_dim)
        if self.attention == "native":
            # The tensor-core kernels read [B, S, heads, D] as it stands and
            # write the output in the layout o_proj reads.
            att = glue.attention(q, k, v, causal=True).view(B, S, cfg.heads * cfg.head_dim)
        else:
            att = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                                 v.transpose(1, 2), is_causal=True,
                                                 enable_gqa=cfg.heads != cfg.kv_heads)
            att = att.transpose(1, 2).reshape(B, S, cfg.heads * cfg.head_dim)
        x, h = glue.add_rms_norm(x, qlora_linear(att, blk.linears["o_proj"],
                                                 blk.adapters["o_proj"]),
                                 blk.post_norm, cfg.rms_eps)
        gu = ("gate_proj", "up_proj")
        g, u = qlora_linears(h, [blk.linears[n] for n in gu], [blk.adapters[n] for n in gu])
        return glue.add_rms_norm(x, qlora_linear(glue.swiglu(g, u), blk.linears["down_proj"],
                                                 blk.adapters["down_proj"]),
                                 next_norm, cfg.rms_eps)

    def hidden(self, ids: torch.Tensor) -> torch.Tensor:
        """The final-normed hidden states: the blocks' residual stream
        (``x += attn(norm(x)); x += mlp(norm(x))``) and the final norm."""
        x = F.embedding(ids, self.embed)
        if not self.blocks:
            return glue.rms_norm(x, self.final_norm, self.cfg.rms_eps)
        h = glue.rms_norm(x, self.blocks[0].input_norm, self.cfg.rms_eps)
        for i, blk in enumerate(self.blocks):
            nxt = self.blocks[i + 1].input_norm if i + 1 < len(self.blocks) else self.final_norm
            x, h = self.block_forward(blk, x, h, nxt)
        return h

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        head = self.embed if self.lm_head is None else self.lm_head
        return h @ head.t()

    def loss(self, ids: torch.Tensor) -> torch.Tensor:
        """Mean next-token cross-entropy (f32) over positions 0..S-2: the
        fused per-position loss kernel, its gradient written over the bf16
        logits in backward."""
        h = self.hidden(ids)[:, :-1]
        z = self.logits(h)
        tgt = ids[:, 1:]
        return glue.cross_entropy(z, tgt, inplace=True).mean()

    def base_nbytes(self) -> int:
        return sum(w.nbytes() for blk in self.blocks for w in blk.linears.values())

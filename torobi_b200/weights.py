"""Parameter names, the dtype vocabulary, and reading published weights.

Names follow the published (Hugging Face) layout the reference's Llama family
declares (lib/torobi/models/llama.rb:255-327): ``model.embed_tokens.weight``,
``model.layers.{i}.input_layernorm.weight``,
``model.layers.{i}.self_attn.{q,k,v,o}_proj.weight`` (and ``.bias`` for the
qwen2 family's q/k/v), ``model.layers.{i}.post_attention_layernorm.weight``,
``model.layers.{i}.mlp.{gate,up,down}_proj.weight``, ``model.norm.weight`` and
``lm_head.weight`` when the head is not tied.  A LoRA pair beside a linear is
``<linear>.lora_A.weight`` [rank, d_in] and ``<linear>.lora_B.weight`` [d_out,
rank] (PEFT's names, lib/torobi/lora.rb:33-34, :63).  A quantized linear's
weight is three tensors, MLX's spelling for a quantized layer:
``<linear>.weight`` (u32 codes), ``<linear>.scales`` and ``<linear>.biases``.

The dtype vocabulary is the reference's (engine/src/tensor.rs:142-170,
lib/torobi/ir/dtype.rb:8) plus ``u32``, which packed codes need.

Loading a published model follows the reference's pretrained source
(engine/src/plan.rs:381-520): each declared parameter is looked up by its
published path, its shape must match, its dtype is converted to the declared
one, a missing path is an error that names it, and the adapter's matrices
are fresh (drawn from the seed) rather than read.  The linears are quantized
as they arrive, on the device: the hook the reference's parameter conversion
(engine/src/plan.rs:499) would call.
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import torch

VOCABULARY: tuple[tuple[str, torch.dtype], ...] = (
    ("f32", torch.float32),
    ("bf16", torch.bfloat16),
    ("i32", torch.int32),
    ("bool", torch.bool),
    ("u32", torch.uint32),
)

ATTENTION = ("q_proj", "k_proj", "v_proj", "o_proj")
MLP = ("gate_proj", "up_proj", "down_proj")
LORA_SUFFIXES = ("lora_A.weight", "lora_B.weight")


def dtype_named(name: str) -> torch.dtype | None:
    """The dtype a name in the vocabulary means (None for an unknown name)."""
    for spelled, dt in VOCABULARY:
        if spelled == name:
            return dt
    return None


def dtype_spelling(dtype: torch.dtype) -> str | None:
    """What the vocabulary calls a dtype (None: it cannot be named, so a
    checkpoint must refuse it)."""
    for spelled, dt in VOCABULARY:
        if dt == dtype:
            return spelled
    return None


def linear_path(layer: int, name: str) -> str:
    scope = "self_attn" if name in ATTENTION else "mlp"
    if name not in ATTENTION and name not in MLP:
        raise ValueError(f"unknown linear {name!r}")
    return f"model.layers.{layer}.{scope}.{name}"


def adapter_paths(layer: int, name: str) -> tuple[str, str]:
    base = linear_path(layer, name)
    return tuple(f"{base}.{s}" for s in LORA_SUFFIXES)  # type: ignore[return-value]


def is_adapter_path(path: str) -> bool:
    """Whether a parameter path is an adapter's own (lib/torobi/lora.rb:106-110)."""
    return any(path.endswith("." + s) for s in LORA_SUFFIXES)


@dataclass(frozen=True)
class Declared:
    """One parameter of a dense published model: its path, shape, dtype."""

    path: str
    shape: tuple[int, ...]
    dtype: str


def published_parameters(cfg) -> list[Declared]:
    """Every parameter a dense published checkpoint of this shape holds, in
    declaration order (embedding, then each layer, then the final norm and
    the head)."""
    out = [Declared("model.embed_tokens.weight", (cfg.vocab, cfg.hidden), "bf16")]
    shapes = cfg.linear_shapes()
    for i in range(cfg.layers):
        out.append(Declared(f"model.layers.{i}.input_layernorm.weight", (cfg.hidden,), "bf16"))
        for name in ATTENTION:
            d_out, d_in = shapes[name]
            out.append(Declared(f"{linear_path(i, name)}.weight", (d_out, d_in), "bf16"))
            if cfg.attention_bias and name != "o_proj":
                out.append(Declared(f"{linear_path(i, name)}.bias", (d_out,), "bf16"))
        out.append(Declared(f"model.layers.{i}.post_attention_layernorm.weight", (cfg.hidden,),
                            "bf16"))
        for name in MLP:
            d_out, d_in = shapes[name]
            out.append(Declared(f"{linear_path(i, name)}.weight", (d_out, d_in), "bf16"))
    out.append(Declared("model.norm.weight", (cfg.hidden,), "bf16"))
    if not cfg.tie_embeddings:
        out.append(Declared("lm_head.weight", (cfg.vocab, cfg.hidden), "bf16"))
    return out


class SafetensorsSource:
    """A published model's file, read tensor by tensor as the model is built."""

    def __init__(self, path: str | Path):
        from safetensors import safe_open

        self.path = Path(path)
        self._f = safe_open(str(self.path), framework="pt", device="cpu")
        self._keys = set(self._f.keys())

    def tensor(self, path: str, shape: tuple[int, ...], dtype: torch.dtype,
               device: torch.device) -> torch.Tensor:
        if path not in self._keys:
            raise KeyError(
                f"{self.path.name} has no parameter {path!r}. If it is meant to be new, "
                "name it as fresh: a parameter that is in no checkpoint has to be said to be "
                "new, which is what tells a typo from a fresh parameter.")
        t = self._f.get_tensor(path)
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"parameter {path!r}: given shape {tuple(t.shape)} is not the "
                             f"declared {tuple(shape)}")
        # Importing is starting somewhere, not resuming: the dtype converts.
        return t.to(device=device).to(dtype)

    def keys(self) -> set[str]:
        return set(self._keys)


def write_dense(path: str | Path, tensors: dict[str, torch.Tensor],
                metadata: dict[str, str] | None = None) -> None:
    """Writes tensors (any device) to one safetensors file."""
    from safetensors.torch import save_file

    save_file({k: v.detach().to("cpu", copy=True).contiguous() for k, v in tensors.items()},
              str(path),
              metadata=metadata)

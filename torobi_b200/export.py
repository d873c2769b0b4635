"""Exporting a QLoRA-trained model: merged into published fp32 weights, or
the adapter on its own.

``export_model`` writes what the reference's export writes for a dense run
(engine/src/export.rs:1-90): one model's parameters under the published names,
fp32, ``{"format": "pt"}`` metadata, in ``model.safetensors``, read back
before it counts.  The reference refuses an adapted run because merging
``W + scale * BA`` "is not built yet" (lib/torobi/export.rb:118-140); here
every adapted linear is merged on the device (``ops.lora_merge``: the
quantized base dequantized as the GEMM sees it, plus the scaled low-rank
product) and the adapter is dropped, so the file is a dense model that
carries what was trained.

``export_adapter`` writes the unmerged pair instead, under PEFT's names
(``base_model.model.<linear>.lora_A.weight`` / ``lora_B.weight``, f32) with an
``adapter_config.json`` giving rank, alpha and the targets.
"""
from __future__ import annotations

import json
from pathlib import Path

import torch

from . import ops
from .weights import ATTENTION, MLP, adapter_paths, linear_path, write_dense


def merged_tensors(model, dtype: torch.dtype = torch.float32) -> dict[str, torch.Tensor]:
    """Every published parameter of the model, adapters merged, on the host."""
    cfg = model.cfg
    out: dict[str, torch.Tensor] = {}

    def put(path, t):
        out[path] = t.to(dtype).cpu()

    put("model.embed_tokens.weight", model.embed)
    for li, blk in enumerate(model.blocks):
        put(f"model.layers.{li}.input_layernorm.weight", blk.input_norm)
        for name in ATTENTION + MLP:
            if name == "gate_proj":
                put(f"model.layers.{li}.post_attention_layernorm.weight", blk.post_norm)
            w = blk.linears[name]
            ad = blk.adapters.get(name)
            merged = ops.lora_merge(w.codes, w.scales, w.biases, w.group, w.bits,
                                    lora_a=None if ad is None else ad.a,
                                    lora_b=None if ad is None else ad.b,
                                    scale=1.0 if ad is None else ad.scale, dtype=dtype)
            out[f"{linear_path(li, name)}.weight"] = merged.cpu()
            del merged
            if w.bias is not None:
                put(f"{linear_path(li, name)}.bias", w.bias)
    put("model.norm.weight", model.final_norm)
    if not cfg.tie_embeddings:
        put("lm_head.weight", model.lm_head)
    return out


def export_model(model, directory, dtype: torch.dtype = torch.float32) -> Path:
    """Writes ``<directory>/model.safetensors`` (adapters merged) and returns
    its path, after reading it back."""
    from safetensors import safe_open

    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    tensors = merged_tensors(model, dtype)
    f = d / "model.safetensors"
    write_dense(f, tensors, metadata={"format": "pt"})
    with safe_open(str(f), framework="pt", device="cpu") as r:
        keys = set(r.keys())
    missing = set(tensors) - keys
    if missing or len(keys) != len(tensors):
        raise RuntimeError(f"the export just written does not read back ({len(keys)} tensors, "
                           f"{len(tensors)} saved; missing {sorted(missing)[:3]})")
    return f


def export_adapter(model, directory) -> Path:
    """Writes the trained pairs, unmerged, as ``adapter_model.safetensors``
    plus ``adapter_config.json``."""
    cfg = model.cfg
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    tensors = {}
    for li, blk in enumerate(model.blocks):
        for name, ad in blk.adapters.items():
            if ad is None:
                continue
            pa, pb = adapter_paths(li, name)
            tensors[f"base_model.model.{pa}"] = ad.a
            tensors[f"base_model.model.{pb}"] = ad.b
    f = d / "adapter_model.safetensors"
    write_dense(f, tensors, metadata={"format": "pt"})
    (d / "adapter_config.json").write_text(json.dumps({
        "peft_type": "LORA", "task_type": "CAUSAL_LM", "r": cfg.lora_rank,
        "lora_alpha": cfg.lora_alpha, "target_modules": list(cfg.lora_targets),
        "lora_dropout": 0.0, "bias": "none"}, indent=2))
    return f

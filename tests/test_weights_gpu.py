"""Quantize-at-load: a published (dense, bf16) safetensors file becomes the
QLoRA model, every block linear quantized on the device as it arrives, codes,
scales and biases bit-exact to the oracle's quantization of the same weights;
norms, embedding and head taken as they are; the adapter fresh.  The
reference's pretrained source rules (engine/src/plan.rs:381-520): a missing
path and a wrong shape are refused, a dtype is converted."""
from __future__ import annotations

import numpy as np
import pytest

from _util import host_bf16, host_u32


def _dense_file(tmp_path, cfg, dtype=None):
    import torch

    from torobi_b200.weights import published_parameters, write_dense

    g = torch.Generator().manual_seed(3)
    tensors = {}
    for d in published_parameters(cfg):
        t = torch.randn(d.shape, generator=g) * (0.02 if len(d.shape) == 2 else 1.0)
        tensors[d.path] = t.to(dtype or torch.bfloat16)
    f = tmp_path / "model.safetensors"
    write_dense(f, tensors, metadata={"format": "pt"})
    return f, tensors


@pytest.mark.gpu
@pytest.mark.parametrize("tied", [True, False])
def test_from_pretrained_quantizes_at_load(cuda, oracle, tmp_path, tied):
    import torch

    from torobi_b200.model import QLoRACausalLM, tiny_config
    from torobi_b200.weights import linear_path

    cfg = tiny_config(tie_embeddings=tied, attention_bias=tied)
    f, dense = _dense_file(tmp_path, cfg)
    model = QLoRACausalLM.from_pretrained(cfg, f, device=cuda, seed=1)
    for li, blk in enumerate(model.blocks):
        for name, w in blk.linears.items():
            src = dense[f"{linear_path(li, name)}.weight"]
            bits = src.view(torch.int16).numpy().view(np.uint16)
            c, s, b = oracle.quantize(bits, cfg.bits, cfg.group)
            assert np.array_equal(host_u32(w.codes), c), (li, name)
            assert np.array_equal(host_bf16(w.scales), s), (li, name)
            assert np.array_equal(host_bf16(w.biases), b), (li, name)
            if w.bias is not None:
                assert torch.equal(w.bias.cpu(), dense[f"{linear_path(li, name)}.bias"])
        assert torch.equal(blk.input_norm.cpu(), dense[f"model.layers.{li}.input_layernorm.weight"])
    assert torch.equal(model.embed.cpu(), dense["model.embed_tokens.weight"])
    assert torch.equal(model.final_norm.cpu(), dense["model.norm.weight"])
    if not tied:
        assert torch.equal(model.lm_head.cpu(), dense["lm_head.weight"])
    # The adapter is fresh: B starts at zero, so the model is the loaded one.
    for ad in model.store.adapters.values():
        assert float(ad.b.abs().max()) == 0.0
    ids = torch.randint(0, cfg.vocab, (2, 16), device=cuda)
    assert torch.isfinite(model.loss(ids))


@pytest.mark.gpu
def test_from_pretrained_converts_f32_and_refuses_mismatches(cuda, tmp_path):
    import torch

    from torobi_b200.model import QLoRACausalLM, tiny_config
    from torobi_b200.weights import write_dense

    cfg = tiny_config()
    f, dense = _dense_file(tmp_path, cfg, dtype=torch.float32)
    model = QLoRACausalLM.from_pretrained(cfg, f, device=cuda)
    assert model.embed.dtype == torch.bfloat16
    assert torch.equal(model.embed.cpu(), dense["model.embed_tokens.weight"].bfloat16())
    missing = dict(dense)
    del missing["model.layers.1.mlp.up_proj.weight"]
    write_dense(tmp_path / "missing.safetensors", missing)
    with pytest.raises(KeyError, match="up_proj"):
        QLoRACausalLM.from_pretrained(cfg, tmp_path / "missing.safetensors", device=cuda)
    wrong = dict(dense)
    wrong["model.norm.weight"] = torch.ones(cfg.hidden + 1)
    write_dense(tmp_path / "wrong.safetensors", wrong)
    with pytest.raises(ValueError, match="model.norm.weight"):
        QLoRACausalLM.from_pretrained(cfg, tmp_path / "wrong.safetensors", device=cuda)

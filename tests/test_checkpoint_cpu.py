"""Host logic of the checkpoint, the dtype vocabulary and the published
names, on CPU tensors (no GPU): the layout and manifest the reference writes
(engine/src/checkpoint.rs), the atomic publish, and the refusals."""
from __future__ import annotations

import json
from types import SimpleNamespace

import pytest
import torch

from torobi_b200 import checkpoint
from torobi_b200.model import QWEN2_5_0_5B, Block, tiny_config
from torobi_b200.qlora import Adapter, QuantizedWeight
from torobi_b200.train import AdamWConfig
from torobi_b200.weights import (dtype_named, dtype_spelling, is_adapter_path, linear_path,
                                 published_parameters)


def test_dtype_vocabulary_round_trips_and_names_u32():
    for name in ("f32", "bf16", "i32", "bool", "u32"):
        assert dtype_spelling(dtype_named(name)) == name
    assert dtype_named("f16") is None and dtype_spelling(torch.float16) is None


def test_published_names_follow_the_llama_layout():
    names = [d.path for d in published_parameters(QWEN2_5_0_5B)]
    # embedding, 24 x (2 norms + 7 weights + 3 q/k/v biases), final norm (tied head)
    assert len(names) == 1 + 24 * 12 + 1
    assert names[:4] == ["model.embed_tokens.weight", "model.layers.0.input_layernorm.weight",
                         "model.layers.0.self_attn.q_proj.weight",
                         "model.layers.0.self_attn.q_proj.bias"]
    assert linear_path(3, "down_proj") == "model.layers.3.mlp.down_proj"
    assert is_adapter_path("model.layers.0.self_attn.q_proj.lora_B.weight")


def _fake(seed=0):
    """A trainer-shaped object over CPU tensors with the attributes the
    checkpoint reads."""
    cfg = tiny_config(layers=1)
    g = torch.Generator().manual_seed(seed)
    total = 0
    layout = {}
    shapes = cfg.linear_shapes()
    for name in cfg.lora_targets:
        d_out, d_in = shapes[name]
        layout[name] = (total, total + cfg.lora_rank * d_in)
        total += cfg.lora_rank * (d_in + d_out)
    params = torch.randn(total, generator=g)
    store = SimpleNamespace(params=params, m=torch.randn(total, generator=g),
                            v=torch.rand(total, generator=g), refresh_bf16=lambda full=False: None)
    blk = Block(torch.ones(cfg.hidden, dtype=torch.bfloat16),
                torch.ones(cfg.hidden, dtype=torch.bfloat16))
    for name, (d_out, d_in) in shapes.items():
        codes = torch.randint(0, 2**31, (d_out, d_in // 8), generator=g).to(torch.uint32)
        sc = torch.randn(d_out, d_in // cfg.group, generator=g).bfloat16()
        bias = torch.zeros(d_out, dtype=torch.bfloat16) if name in ("q_proj", "k_proj",
                                                                     "v_proj") else None
        blk.linears[name] = QuantizedWeight(codes, sc, sc.clone(), cfg.bits, cfg.group, bias)
        ad = None
        if name in layout:
            oa, ob = layout[name]
            ad = Adapter(name, cfg.lora_rank, 2.0,
                         params[oa:oa + cfg.lora_rank * d_in].view(cfg.lora_rank, d_in),
                         params[ob:ob + d_out * cfg.lora_rank].view(d_out, cfg.lora_rank),
                         None, None, None, None, None)
        blk.adapters[name] = ad
    model = SimpleNamespace(cfg=cfg, embed=torch.randn(cfg.vocab, cfg.hidden, generator=g).bfloat16(),
                            final_norm=torch.ones(cfg.hidden, dtype=torch.bfloat16), lm_head=None,
                            blocks=[blk], store=store)
    return SimpleNamespace(model=model, opt=AdamWConfig(lr=1e-3), t=7, steps=9,
                           settle=lambda: float("nan"))


def test_save_read_restore_round_trip(tmp_path):
    tr = _fake(0)
    d = checkpoint.save(tr, tmp_path / "c", seed=3, run={"batch": 12})
    assert sorted(p.name for p in d.iterdir()) == ["graph.json", "manifest.json",
                                                   "optimizer.safetensors",
                                                   "parameters.safetensors", "random.safetensors"]
    man = checkpoint.read_manifest(d)
    assert man["schema_version"] == 2 and man["optimizer_steps"] == 7 and man["step"] == 9
    assert man["optimizer"]["kind"] == "adamw" and man["seed"] == 3
    dtypes = {e["path"]: e["dtype"] for e in man["parameters"]}
    assert dtypes["model.layers.0.self_attn.q_proj.weight"] == "u32"
    assert dtypes["model.layers.0.self_attn.q_proj.lora_A.weight"] == "f32"
    trained = [e["path"] for e in man["parameters"] if e["trained"]]
    assert trained and all(is_adapter_path(p) for p in trained)
    other = _fake(1)
    other.t = other.steps = 0
    checkpoint.restore(other, d)
    assert torch.equal(other.model.store.params, tr.model.store.params)
    assert torch.equal(other.model.store.m, tr.model.store.m)
    assert torch.equal(other.model.blocks[0].linears["up_proj"].codes,
                       tr.model.blocks[0].linears["up_proj"].codes)
    assert other.t == 7 and other.steps == 9


def test_refusals(tmp_path):
    tr = _fake(0)
    d = checkpoint.save(tr, tmp_path / "c")
    # another optimizer
    other = _fake(0)
    other.opt = AdamWConfig(lr=5e-4)
    with pytest.raises(ValueError, match="different optimizer"):
        checkpoint.restore(other, d)
    # a description that is not the one the digest names
    (d / "graph.json").write_text("{}")
    with pytest.raises(ValueError, match="digest"):
        checkpoint.read(d)
    # another schema
    d2 = checkpoint.save(tr, tmp_path / "c2")
    man = json.loads((d2 / "manifest.json").read_text())
    man["schema_version"] = 1
    (d2 / "manifest.json").write_text(json.dumps(man))
    with pytest.raises(ValueError, match="schema"):
        checkpoint.read(d2)
    # nothing was touched by a refused restore
    assert torch.equal(other.model.store.params, _fake(0).model.store.params)

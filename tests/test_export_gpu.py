"""Export after QLoRA training: merged into a dense fp32 model under the
published names (every adapted linear = dequantized base + scale * B A,
bit-exact to the oracle; the others dequantized; norms, embedding and head
as they are), and the adapter alone under PEFT's names."""
from __future__ import annotations

import json

import numpy as np
import pytest

from _util import host_bf16, host_u32


@pytest.mark.gpu
def test_export_model_merges_the_adapter(cuda, oracle, tmp_path):
    import torch
    from safetensors.torch import load_file

    from torobi_b200.export import export_model
    from torobi_b200.model import QLoRACausalLM, tiny_config
    from torobi_b200.train import AdamWConfig, Trainer
    from torobi_b200.weights import linear_path, published_parameters

    cfg = tiny_config(tie_embeddings=False)
    model = QLoRACausalLM(cfg, device=cuda, seed=2)
    tr = Trainer(model, AdamWConfig(lr=1e-2), micro_batch=2)
    ids = torch.randint(0, cfg.vocab, (2, 32), device=cuda)
    for _ in range(2):
        tr.step(ids)
    f = export_model(model, tmp_path / "out")
    got = load_file(str(f))
    assert set(got) == {d.path for d in published_parameters(cfg)}
    assert all(t.dtype == torch.float32 for t in got.values())
    for li, blk in enumerate(model.blocks):
        for name, w in blk.linears.items():
            ad = blk.adapters[name]
            c, s, b = host_u32(w.codes), host_bf16(w.scales), host_bf16(w.biases)
            if ad is None:
                want = oracle.lora_merge(c, s, b, w.bits, w.group)
            else:
                assert float(ad.b.abs().max()) > 0.0  # trained, so the merge matters
                want = oracle.lora_merge(c, s, b, w.bits, w.group, ad.a.cpu().numpy(),
                                         ad.b.cpu().numpy(), ad.scale)
            assert np.array_equal(got[f"{linear_path(li, name)}.weight"].numpy(), want)
    assert torch.equal(got["lm_head.weight"], model.lm_head.float().cpu())


@pytest.mark.gpu
def test_export_adapter_writes_peft_names(cuda, tmp_path):
    import torch
    from safetensors.torch import load_file

    from torobi_b200.export import export_adapter
    from torobi_b200.model import QLoRACausalLM, tiny_config

    cfg = tiny_config()
    model = QLoRACausalLM(cfg, device=cuda)
    f = export_adapter(model, tmp_path / "adapter")
    got = load_file(str(f))
    conf = json.loads((tmp_path / "adapter" / "adapter_config.json").read_text())
    assert conf["r"] == cfg.lora_rank and conf["target_modules"] == list(cfg.lora_targets)
    assert len(got) == 2 * cfg.layers * len(cfg.lora_targets)
    key = "base_model.model.model.layers.1.self_attn.v_proj.lora_A.weight"
    assert torch.equal(got[key], model.store.adapters["layers.1.v_proj"].a.cpu())

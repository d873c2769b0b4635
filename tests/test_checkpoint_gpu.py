"""Checkpoint and resume of a QLoRA run (the reference's layout,
engine/src/checkpoint.rs): everything restored bit for bit, the next step the
same as a run that never stopped, and a checkpoint of another model or
optimizer refused before anything is touched."""
from __future__ import annotations

import json

import pytest


def _run(cuda, seed=0, lr=1e-3):
    import torch

    from torobi_b200.model import QLoRACausalLM, tiny_config
    from torobi_b200.train import AdamWConfig, Trainer

    cfg = tiny_config()
    model = QLoRACausalLM(cfg, device=cuda, seed=seed)
    tr = Trainer(model, AdamWConfig(lr=lr, weight_decay=0.01), micro_batch=2)
    g = torch.Generator(device=cuda).manual_seed(9)
    ids = torch.randint(0, cfg.vocab, (4, 32), device=cuda, generator=g)
    return model, tr, ids


@pytest.mark.gpu
def test_save_restore_resumes_the_same_run(cuda, tmp_path):
    import torch

    from torobi_b200 import checkpoint

    model, tr, ids = _run(cuda)
    for _ in range(2):
        tr.step(ids)
        tr.settle()
    d = checkpoint.save(tr, tmp_path / "ckpt", seed=0, run={"epoch": 1})
    assert not (tmp_path / "ckpt.writing").exists()
    saved = {k: v.clone() for k, v in (("p", model.store.params), ("m", model.store.m),
                                       ("v", model.store.v))}
    want_loss = float(tr.step(ids))
    want_p = model.store.params.clone()

    # Another run, from another seed: everything it holds is replaced.
    model2, tr2, _ = _run(cuda, seed=5)
    m = checkpoint.restore(tr2, d)
    assert m["run"] == {"epoch": 1} and tr2.t == 2 and tr2.steps == 2
    assert torch.equal(model2.store.params, saved["p"])
    assert torch.equal(model2.store.m, saved["m"])
    assert torch.equal(model2.store.v, saved["v"])
    for b1, b2 in zip(model.blocks, model2.blocks):
        for name in b1.linears:
            assert torch.equal(b1.linears[name].codes, b2.linears[name].codes)
    got_loss = float(tr2.step(ids))
    assert abs(got_loss - want_loss) <= 1e-5 * abs(want_loss)
    assert torch.allclose(model2.store.params, want_p, rtol=0, atol=1e-6)


@pytest.mark.gpu
def test_restore_refuses_another_model_or_optimizer(cuda, tmp_path):
    from torobi_b200 import checkpoint
    from torobi_b200.model import QLoRACausalLM, tiny_config
    from torobi_b200.train import AdamWConfig, Trainer

    model, tr, ids = _run(cuda)
    d = checkpoint.save(tr, tmp_path / "ckpt")
    other = Trainer(QLoRACausalLM(tiny_config(lora_rank=16), device=cuda), AdamWConfig(lr=1e-3))
    with pytest.raises(ValueError, match="another model"):
        checkpoint.restore(other, d)
    _, tr3, _ = _run(cuda, lr=2e-3)
    with pytest.raises(ValueError, match="different optimizer"):
        checkpoint.restore(tr3, d)
    # A manifest that lies about a shape is refused when read.
    mf = d / "manifest.json"
    man = json.loads(mf.read_text())
    man["parameters"][1]["shape"] = [7]
    mf.write_text(json.dumps(man))
    with pytest.raises(ValueError, match="manifest"):
        checkpoint.restore(tr, d)


@pytest.mark.gpu
def test_save_replaces_an_older_checkpoint_whole(cuda, tmp_path):
    from torobi_b200 import checkpoint

    model, tr, ids = _run(cuda)
    d = checkpoint.save(tr, tmp_path / "ckpt")
    tr.step(ids)
    tr.settle()
    checkpoint.save(tr, d)
    assert checkpoint.read_manifest(d)["optimizer_steps"] == 1
    assert sorted(p.name for p in tmp_path.iterdir()) == ["ckpt"]


@pytest.mark.gpu
def test_save_right_after_a_skipped_step_counts_only_taken_steps(cuda, tmp_path):
    """A step whose gradient norm is not finite is skipped on the device
    (engine/src/state.rs:360-370); a checkpoint written straight after it,
    before anything read the norm back, records the steps actually taken."""
    from torobi_b200 import checkpoint

    model, tr, ids = _run(cuda)
    tr.step(ids)
    tr.settle()
    a = next(iter(model.store.adapters.values()))
    a.a[0, 0] = float("nan")  # the next loss and gradients are NaN
    model.store.refresh_bf16(full=True)
    tr.step(ids)  # launched, not settled
    d = checkpoint.save(tr, tmp_path / "ckpt")
    assert checkpoint.read_manifest(d)["optimizer_steps"] == 1
    assert tr.t == 1

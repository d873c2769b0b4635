"""The QLoRA causal LM end to end on the GPU: the loss of the bf16 model
through the quantized kernels against an f32 torch restatement of the same
graph on the same dequantized weights, the adapter's gradients against that
restatement's autograd, the adapter starting as the base model, and a few
steps that lower the loss while the base stays untouched."""
from __future__ import annotations

import math

import pytest


def _f32_reference_loss(model, ids):
    """The same architecture in f32 torch on the dequantized weights."""
    import torch
    import torch.nn.functional as F

    import torobi_b200 as tq
    from torobi_b200.model import apply_rope

    cfg = model.cfg

    def lin(x, w, ad):
        wd = tq.dequantize(w.codes, w.scales, w.biases, w.group, w.bits).float()
        y = x @ wd.t()
        if w.bias is not None:
            y = y + w.bias.float()
        if ad is not None:
            y = y + ((x @ ad.a.t()) @ ad.b.t()) * ad.scale
        return y

    def norm(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * w.float()

    x = F.embedding(ids, model.embed.float())
    B, S, _ = x.shape
    cos, sin = model._rope(S)
    for blk in model.blocks:
        h = norm(x, blk.input_norm)
        q = lin(h, blk.linears["q_proj"], blk.adapters["q_proj"]).view(B, S, cfg.heads, -1)
        k = lin(h, blk.linears["k_proj"], blk.adapters["k_proj"]).view(B, S, cfg.kv_heads, -1)
        v = lin(h, blk.linears["v_proj"], blk.adapters["v_proj"]).view(B, S, cfg.kv_heads, -1)
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        rep = cfg.heads // cfg.kv_heads
        k, v = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
        att = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + lin(att.transpose(1, 2).reshape(B, S, -1), blk.linears["o_proj"],
                    blk.adapters["o_proj"])
        h = norm(x, blk.post_norm)
        g = lin(h, blk.linears["gate_proj"], blk.adapters["gate_proj"])
        u = lin(h, blk.linears["up_proj"], blk.adapters["up_proj"])
        x = x + lin(F.silu(g) * u, blk.linears["down_proj"], blk.adapters["down_proj"])
    h = norm(x, model.final_norm)[:, :-1]
    head = model.embed if model.lm_head is None else model.lm_head
    z = h @ head.float().t()
    return F.cross_entropy(z.reshape(-1, z.shape[-1]), ids[:, 1:].reshape(-1))


@pytest.mark.gpu
@pytest.mark.parametrize("tied", [True, False])
def test_loss_matches_f32_reference(cuda, tied):
    """A full step's loss within 1e-3 relative of the f32 restatement."""
    import torch

    from torobi_b200.model import QLoRACausalLM, tiny_config

    cfg = tiny_config(tie_embeddings=tied, attention_bias=tied, lora_rank=16, lora_alpha=32.0,
                      lora_targets=("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj",
                                    "up_proj", "down_proj"))
    model = QLoRACausalLM(cfg, cuda, seed=3)
    for ad in model.store.adapters.values():  # non-zero B so the adapter contributes
        ad.b.normal_(0.0, 0.02)
    model.store.refresh_bf16(full=True)
    g = torch.Generator(device=cuda)
    g.manual_seed(0)
    ids = torch.randint(0, cfg.vocab, (4, 128), generator=g, device=cuda)
    with torch.no_grad():
        got = float(model.loss(ids))
        want = float(_f32_reference_loss(model, ids))
    assert abs(got - want) / want < 1e-3, (got, want)
    assert abs(want - math.log(cfg.vocab)) < 2.0  # near uniform at random init


@pytest.mark.gpu
def test_native_attention_loss_and_gradients(cuda):
    """The model with this package's attention kernels (attention="native"):
    the loss within 1e-3 relative of the f32 restatement, and the adapters'
    gradients against that restatement's autograd by the bar of the model
    gradient test (relative norm error < 5e-2, cosine > 0.999)."""
    import torch

    from torobi_b200.model import QLoRACausalLM, tiny_config

    cfg = tiny_config(heads=8, kv_heads=2, head_dim=64, hidden=512, lora_rank=16,
                      lora_alpha=32.0, lora_targets=("q_proj", "k_proj", "v_proj", "o_proj"))
    g = torch.Generator(device=cuda)
    g.manual_seed(1)
    ids = torch.randint(0, cfg.vocab, (2, 384), generator=g, device=cuda)
    model = QLoRACausalLM(cfg, cuda, seed=4, attention="native")
    for ad in model.store.adapters.values():
        ad.b.normal_(0.0, 0.02)
    model.store.refresh_bf16(full=True)
    model.store.zero_grad()
    loss = model.loss(ids)
    loss.backward()
    with torch.no_grad():
        want = float(_f32_reference_loss(model, ids))
    assert abs(float(loss) - want) / want < 1e-3, (float(loss), want)
    got = {n: (ad.ga.clone(), ad.gb.clone()) for n, ad in model.store.adapters.items()}
    leaves = {}
    for n, ad in model.store.adapters.items():
        a = ad.a.detach().clone().requires_grad_()
        b = ad.b.detach().clone().requires_grad_()
        leaves[n] = (a, b)
        ad.a, ad.b = a, b
    _f32_reference_loss(model, ids).backward()
    for n, (a, b) in leaves.items():
        for mine, ref in ((got[n][0], a.grad), (got[n][1], b.grad)):
            err = ((mine - ref).norm() / ref.norm()).item()
            cos = torch.nn.functional.cosine_similarity(mine.flatten(), ref.flatten(), dim=0).item()
            assert err < 5e-2 and cos > 0.999, (n, err, cos)


def _random_adapters(model, std):
    """Non-zero B so the adapter contributes to the loss."""
    for ad in model.store.adapters.values():
        ad.b.normal_(0.0, std)
    model.store.refresh_bf16(full=True)


@pytest.mark.gpu
def test_loss_matches_f32_reference_llama3_8b_widths(cuda):
    """The Llama-3-8B-shaped model's exact widths (hidden 4096, 32/8 heads of
    128, SwiGLU 14336, untied 128256 vocabulary, theta 5e5, LoRA r16 alpha 32
    on all seven projections, 4-bit g64), two layers deep, on 2 x 2048 tokens:
    the loss within 1e-3 relative of the f32 restatement."""
    import dataclasses

    import torch

    from torobi_b200.model import LLAMA3_8B, QLoRACausalLM

    cfg = dataclasses.replace(LLAMA3_8B, layers=2)
    model = QLoRACausalLM(cfg, cuda, seed=21)
    _random_adapters(model, 0.01)
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    ids = torch.randint(0, cfg.vocab, (2, 2048), generator=g, device=cuda)
    with torch.no_grad():
        got = float(model.loss(ids))
        want = float(_f32_reference_loss(model, ids))
    del model
    torch.cuda.empty_cache()
    assert abs(got - want) / want < 1e-3, (got, want)


@pytest.mark.gpu
def test_loss_matches_f32_reference_qwen2_5_0_5b(cuda):
    """The Qwen2.5-0.5B-shaped model whole: 24 layers, hidden 896, 14/2 heads
    of 64, SwiGLU 4864, tied 151936 vocabulary, q/k/v biases, theta 1e6, LoRA
    r8 alpha 16 on q and v, 4-bit g64; batch 8 x 512: the loss within 1e-3
    relative of the f32 restatement."""
    import torch

    from torobi_b200.model import QWEN2_5_0_5B, QLoRACausalLM

    cfg = QWEN2_5_0_5B
    model = QLoRACausalLM(cfg, cuda, seed=22)
    _random_adapters(model, 0.01)
    for blk in model.blocks:  # non-zero q/k/v biases so they count
        for name in ("q_proj", "k_proj", "v_proj"):
            blk.linears[name].bias.normal_(0.0, 0.02)
    g = torch.Generator(device=cuda)
    g.manual_seed(6)
    ids = torch.randint(0, cfg.vocab, (8, 512), generator=g, device=cuda)
    with torch.no_grad():
        got = float(model.loss(ids))
        want = float(_f32_reference_loss(model, ids))
    del model
    torch.cuda.empty_cache()
    assert abs(got - want) / want < 1e-3, (got, want)


@pytest.mark.gpu
def test_adapter_gradients_match_f32_reference(cuda):
    """bf16 activations against an f32 graph: compared norm-wise (a few bf16
    roundings through attention and the norms separate the two); the per-op
    gradients are held to 1e-2 by the kernel parity tests."""
    import torch

    from torobi_b200.model import QLoRACausalLM, tiny_config

    cfg = tiny_config(lora_targets=("q_proj", "v_proj", "down_proj"))
    model = QLoRACausalLM(cfg, cuda, seed=5)
    for ad in model.store.adapters.values():
        ad.b.normal_(0.0, 0.05)
    model.store.refresh_bf16(full=True)
    g = torch.Generator(device=cuda)
    g.manual_seed(1)
    ids = torch.randint(0, cfg.vocab, (2, 256), generator=g, device=cuda)
    model.store.zero_grad()
    model.loss(ids).backward()
    got = {n: (ad.ga.clone(), ad.gb.clone()) for n, ad in model.store.adapters.items()}
    leaves = {}
    for n, ad in model.store.adapters.items():
        a = ad.a.detach().clone().requires_grad_()
        b = ad.b.detach().clone().requires_grad_()
        leaves[n] = (a, b)
        ad.a, ad.b = a, b
    _f32_reference_loss(model, ids).backward()
    for n, (a, b) in leaves.items():
        for mine, ref in ((got[n][0], a.grad), (got[n][1], b.grad)):
            err = ((mine - ref).norm() / ref.norm()).item()
            cos = torch.nn.functional.cosine_similarity(mine.flatten(), ref.flatten(), dim=0).item()
            assert err < 5e-2 and cos > 0.999, (n, err, cos)


@pytest.mark.gpu
def test_zero_b_starts_as_the_base_model_and_training_moves_only_the_adapter(cuda):
    """test/lora_test.rb:140-168: adapted == base at step 0; after steps the
    base is byte-for-byte unchanged and the loss on the batch falls."""
    import torch

    from torobi_b200.model import QLoRACausalLM, tiny_config
    from torobi_b200.train import AdamWConfig, Trainer

    cfg = tiny_config()
    model = QLoRACausalLM(cfg, cuda, seed=7)
    g = torch.Generator(device=cuda)
    g.manual_seed(2)
    ids = torch.randint(0, cfg.vocab, (8, 64), generator=g, device=cuda)
    with torch.no_grad():
        h_adapted = model.hidden(ids)
        kept = [blk.adapters for blk in model.blocks]
        for blk in model.blocks:
            blk.adapters = {k: None for k in blk.adapters}
        h_base = model.hidden(ids)
        for blk, ad in zip(model.blocks, kept):
            blk.adapters = ad
    assert torch.equal(h_adapted, h_base)
    base_before = [w.codes.clone() for blk in model.blocks for w in blk.linears.values()]
    tr = Trainer(model, AdamWConfig(lr=2e-3), micro_batch=4)
    losses = []
    for _ in range(12):
        losses.append(float(tr.step(ids)))
        tr.settle()
    assert tr.t == 12
    assert losses[-1] < losses[0] - 0.05, losses
    base_after = [w.codes for blk in model.blocks for w in blk.linears.values()]
    assert all(torch.equal(a, b) for a, b in zip(base_before, base_after))


@pytest.mark.gpu
def test_graph_replayed_steps_match_eager_steps(cuda):
    """Trainer(graph=True) replays the forward/backward as a CUDA graph: the
    same losses and parameters as eager steps (to the atomics' summation
    order of the LoRA gradients), a new batch shape captured on its own."""
    import torch

    from torobi_b200.model import QLoRACausalLM, tiny_config
    from torobi_b200.train import AdamWConfig, Trainer

    cfg = tiny_config()
    g = torch.Generator(device=cuda).manual_seed(4)
    batches = [torch.randint(0, cfg.vocab, (4, 32), device=cuda, generator=g) for _ in range(3)]
    runs = []
    for graph in (False, True):
        model = QLoRACausalLM(cfg, device=cuda, seed=11)
        tr = Trainer(model, AdamWConfig(lr=1e-3), micro_batch=2, graph=graph)
        losses = [float(tr.step(b)) for b in batches]
        losses.append(float(tr.step(batches[0][:2])))  # another shape
        runs.append((losses, model.store.params.clone()))
    (l0, p0), (l1, p1) = runs
    assert all(abs(a - b) <= 1e-5 * abs(a) for a, b in zip(l0, l1)), (l0, l1)
    assert torch.allclose(p0, p1, rtol=0, atol=1e-5)


_PDL_SCRIPT = r"""
import sys
sys.path.insert(0, sys.argv[1])
import torch
from torobi_b200.model import QLoRACausalLM, tiny_config
from torobi_b200.train import AdamWConfig, Trainer
cuda = torch.device("cuda", 0)
# Wide enough that the GEMMs run on CTA pairs and the small-token kernel is
# not used: 2048 tokens, hidden 1024, seven adapted projections.
cfg = tiny_config(vocab=4096, hidden=1024, intermediate=2816, heads=8, kv_heads=2,
                  head_dim=128, attention_bias=False, lora_rank=16, lora_alpha=32.0,
                  lora_targets=("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj",
                                "up_proj", "down_proj"))
g = torch.Generator(device=cuda).manual_seed(5)
batches = [torch.randint(0, cfg.vocab, (4, 512), device=cuda, generator=g) for _ in range(3)]
# The native attention: its backward is deterministic, as every other kernel
# of the step but the adapter gradients' atomics.
model = QLoRACausalLM(cfg, device=cuda, seed=13, attention="native")
tr = Trainer(model, AdamWConfig(lr=1e-3), micro_batch=2)
# Losses and adapter gradients of two batches on the initial adapters (with
# B nonzero so every branch carries signal), then one optimizer step.
with torch.no_grad():
    model.store.params.normal_(0.0, 0.02, generator=torch.Generator(device=cuda).manual_seed(6))
model.store.refresh_bf16(full=True)
out = {"losses": [], "grads": []}
for b in batches[:2]:
    model.store.zero_grad()
    loss = model.loss(b)
    loss.backward()
    out["losses"].append(float(loss))
    out["grads"].append(model.store.grads.cpu().clone())
out["step_loss"] = float(tr.step(batches[2]))
torch.save(out, sys.argv[2])
"""


@pytest.mark.gpu
def test_steps_match_without_programmatic_dependent_launch(tmp_path):
    """Every kernel of the step waits on its predecessor (griddepcontrol)
    before touching memory, so launching with programmatic dependent launch
    (the default) or without it (TQ_PDL=0, read once per process, hence the
    child processes) gives the same losses, and the same adapter gradients
    to the summation order of their atomics."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    import torch

    root = str(Path(__file__).resolve().parent.parent)
    runs = []
    for pdl in ("1", "0"):
        out = tmp_path / f"pdl{pdl}.pt"
        res = subprocess.run([sys.executable, "-c", _PDL_SCRIPT, root, str(out)],
                             capture_output=True, text=True, timeout=600,
                             env={**os.environ, "TQ_PDL": pdl})
        assert res.returncode == 0, res.stderr[-2000:]
        runs.append(torch.load(out))
    a, b = runs
    # The forward has no atomics: the same losses.  The adapter gradients
    # differ only by the summation order of their atomics (a race would
    # show as errors of the order of the values themselves).
    assert a["losses"] == b["losses"], (a["losses"], b["losses"])
    for ga, gb in zip(a["grads"], b["grads"]):
        assert ((ga - gb).norm() / ga.norm()).item() < 1e-5
    assert abs(a["step_loss"] - b["step_loss"]) <= 1e-5 * abs(a["step_loss"])


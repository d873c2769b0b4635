"""Data parallelism on two GPUs: the NCCL allreduce of the LoRA gradients
through the library's C ABI.  Two ranks, each stepping on half of a fixed
global batch, must end with identical adapters equal (to f32 rounding) to one
process stepping on the whole batch with the same micro-batch size.

Skipped where fewer than two GPUs are visible (a one-GPU box cannot run it);
the host-side logic is covered on CPU ranks in test_dp_cpu.py."""
from __future__ import annotations

import os
import subprocess
import sys
import tempfile
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent


@pytest.mark.gpu
def test_two_ranks_match_one_process(cuda):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from torobi_b200.model import QLoRACausalLM, tiny_config
    from torobi_b200.train import AdamWConfig, Trainer

    with tempfile.TemporaryDirectory() as d:
        out = Path(d) / "rank0.pt"
        env = dict(os.environ, TQ_DP_OUT=str(out), NCCL_NVLS_ENABLE="0")
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
               "--master-addr=127.0.0.1", "--master-port=29533", str(HERE / "dp_gpu_worker.py")]
        r = subprocess.run(["timeout", "-k", "30", "240", *cmd], env=env, capture_output=True,
                           text=True)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
        got = torch.load(out)
    assert got["same"], "ranks ended with different adapters"
    cfg = tiny_config(lora_targets=("q_proj", "v_proj", "down_proj"))
    model = QLoRACausalLM(cfg, cuda, seed=11)
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    ids = torch.randint(0, cfg.vocab, (8, 128), generator=g, device=cuda)
    tr = Trainer(model, AdamWConfig(lr=1e-2), micro_batch=2)
    losses = []
    for _ in range(2):
        losses.append(float(tr.step(ids)))
        tr.settle()
    assert abs(losses[0] - got["losses"][0]) / losses[0] < 1e-4
    assert abs(losses[1] - got["losses"][1]) / losses[1] < 1e-3
    err = (model.store.params.cpu() - got["params"]).abs().max().item()
    scale = model.store.params.abs().max().item()
    assert err <= 1e-3 * scale, err

"""Host-side logic of the data-parallel step, on CPU ranks over gloo.

Two ranks each take their shard of a global batch, accumulate micro-batch
gradients, sum them with an allreduce and apply the oracle's AdamW with the
trainer's gradient scale; the result must equal one process taking the whole
batch, and both ranks must hold identical parameters."""
from __future__ import annotations

import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest


def test_batch_plan():
    from torobi_b200.train import grad_scale, micro_batches, shard_rows

    assert shard_rows(32, 8, 3) == (12, 16)
    assert micro_batches(8, 4) == [(0, 4), (4, 8)]
    assert grad_scale(8, 2) == 1 / 16
    with pytest.raises(ValueError):
        shard_rows(30, 8, 0)
    with pytest.raises(ValueError):
        micro_batches(6, 4)


def _grads(w, xs, ys):
    pred = xs @ w
    d = 2.0 * (pred - ys) / len(ys)
    return (xs.T @ d).astype(np.float32)


def _worker(rank, world, init_file, out_dir):
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    from oracle import oracle as O
    from torobi_b200.train import grad_scale, micro_batches, shard_rows

    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    rng = np.random.default_rng(0)
    xs = rng.standard_normal((16, 5)).astype(np.float32)
    ys = rng.standard_normal(16).astype(np.float32)
    w = np.zeros(5, np.float32)
    m = np.zeros(5, np.float32)
    v = np.zeros(5, np.float32)
    lo, hi = shard_rows(16, world, rank)
    parts = micro_batches(hi - lo, 2)
    for t in range(1, 4):
        g = np.zeros(5, np.float32)
        for a, b in parts:  # each micro-batch gradient is of its own mean loss
            g += _grads(w, xs[lo + a:lo + b], ys[lo + a:lo + b])
        gt = torch.from_numpy(g)
        dist.all_reduce(gt)
        g = gt.numpy() * np.float32(grad_scale(world, len(parts)))
        w, m, v = O.adamw_step(w, g, m, v, t, lr=0.1)
    np.save(Path(out_dir) / f"w{rank}.npy", w)
    dist.destroy_process_group()


def test_two_gloo_ranks_match_one_process():
    import torch.multiprocessing as mp

    from oracle import oracle as O

    with tempfile.TemporaryDirectory() as d:
        init = os.path.join(d, "init")
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_worker, args=(r, 2, init, d)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        w0 = np.load(os.path.join(d, "w0.npy"))
        w1 = np.load(os.path.join(d, "w1.npy"))
    assert np.array_equal(w0, w1)
    rng = np.random.default_rng(0)
    xs = rng.standard_normal((16, 5)).astype(np.float32)
    ys = rng.standard_normal(16).astype(np.float32)
    w = np.zeros(5, np.float32)
    m = np.zeros(5, np.float32)
    v = np.zeros(5, np.float32)
    for t in range(1, 4):
        w, m, v = O.adamw_step(w, _grads(w, xs, ys), m, v, t, lr=0.1)
    np.testing.assert_allclose(w0, w, rtol=1e-5, atol=1e-6)

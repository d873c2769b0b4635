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


def _gate_worker(rank, world, init, out_dir, fail_rank, timeout):
    import time

    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    from torobi_b200.train import RankLost, StepGate

    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    gate = StepGate(dist.distributed_c10d._get_default_store(), rank, world, timeout=timeout)
    result = "ok"
    t0 = time.monotonic()
    try:
        for step in range(3):
            if rank == fail_rank and step == 1:
                raise RuntimeError("injected failure before step 1's collective")
            gate.wait(step)
            t = torch.ones(1)
            dist.all_reduce(t)
            assert t.item() == world
    except RankLost:
        result = f"lost {time.monotonic() - t0:.2f}"
    except RuntimeError:
        result = "raised"
    (Path(out_dir) / f"r{rank}.txt").write_text(result)
    os._exit(0)  # no teardown handshake with a rank that is gone


def _free_port():
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("store", ["file", "tcp"])
@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_step_gate_reports_a_lost_rank_before_the_collective(store, fail_rank):
    """Three steps on two gloo ranks, each step's collective behind the gate.
    With every rank alive all steps run; when rank 1 raises before step 1,
    rank 0 learns it on the host (RankLost after the gate's 2 s) instead of
    waiting in the collective."""
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        init = f"file://{os.path.join(d, 'init')}" if store == "file" else \
            f"tcp://127.0.0.1:{_free_port()}"
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_gate_worker, args=(r, 2, init, d, fail_rank, 2.0))
                 for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(90)
            if p.exitcode is None:
                p.kill()
            assert p.exitcode == 0
        r0 = (Path(d) / "r0.txt").read_text()
        r1 = (Path(d) / "r1.txt").read_text()
    if fail_rank < 0:
        assert (r0, r1) == ("ok", "ok")
    else:
        assert r1 == "raised"
        assert r0.startswith("lost"), r0
        assert float(r0.split()[1]) < 30.0


def test_step_gate_alone():
    import torch.distributed as dist

    from torobi_b200.train import RankLost, StepGate

    store = dist.HashStore()
    StepGate(store, 0, 1, timeout=0.1).wait(0)  # one rank: nothing to wait for
    gate = StepGate(store, 0, 2, timeout=0.2)
    with pytest.raises(RankLost, match="1 of 2 ranks did not reach step 5"):
        gate.wait(5)
    store.add(gate.key(6), 1)  # the other rank got there first
    gate.wait(6)
    with pytest.raises(ValueError):
        StepGate(store, 0, 2, timeout=0)


def test_step_gate_generations_and_key_cleanup():
    """Each attempt's gates take a fresh generation, so arrivals counted by an
    earlier attempt (e.g. before a restore) never open a later attempt's gate;
    a step's key goes once the next step's gate has passed."""
    import torch.distributed as dist

    from torobi_b200.train import RankLost, StepGate

    store = dist.HashStore()
    g0, g1 = StepGate(store, 0, 2, timeout=0.2), StepGate(store, 1, 2, timeout=0.2)
    assert g0.generation == g1.generation == 0
    store.add(g1.key(0), 1)
    g0.wait(0)
    store.add(g1.key(1), 1)
    g0.wait(1)
    assert not store.check([g0.key(0)]) and store.check([g0.key(1)])
    # A second attempt in the same store, at step counts the first one used.
    h0, h1 = StepGate(store, 0, 2, timeout=0.2), StepGate(store, 1, 2, timeout=0.2)
    assert h0.generation == h1.generation == 1
    with pytest.raises(RankLost):
        h0.wait(1)  # the first attempt's two arrivals at step 1 do not count


class _GlooReduce:
    """The trainer's reduce interface over gloo: launch, then watch."""

    def __init__(self, rank):
        self.rank, self.works, self.aborted = rank, [], False

    def __call__(self, t):
        import torch.distributed as dist

        self.works.append(dist.all_reduce(t, async_op=True))

    def watch(self, timeout):
        from torobi_b200.train import RankLost, wait_collective

        def error():
            for w in self.works:
                if w.is_completed() and not w.is_success():
                    return "gloo work failed"
            return None

        try:
            wait_collective(lambda: all(w.is_completed() for w in self.works), error, timeout,
                            self.rank, "the gradient allreduce")
        except RankLost:
            self.aborted = True
            raise
        self.works.clear()


def _collective_worker(rank, world, init, out_dir, die_after_gate):
    import time

    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    from torobi_b200.train import RankLost, StepGate

    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    gate = StepGate(dist.distributed_c10d._get_default_store(), rank, world, timeout=2.0)
    red = _GlooReduce(rank)
    result = "ok"
    t0 = time.monotonic()
    try:
        for step in range(3):
            gate.wait(step)
            if rank == 1 and step == die_after_gate:
                (Path(out_dir) / "r1.txt").write_text("died")
                os._exit(0)  # past the gate, before its allreduce
            t = torch.ones(4)
            red(t)
            red.watch(gate.timeout)
            assert t[0].item() == world
    except RankLost:
        result = f"lost {time.monotonic() - t0:.2f} aborted={red.aborted}"
    (Path(out_dir) / f"r{rank}.txt").write_text(result)
    os._exit(0)


@pytest.mark.parametrize("die_after_gate", [-1, 1])
def test_a_rank_lost_after_the_gate_is_caught_in_the_collective_wait(die_after_gate):
    """Rank 1 checks in at step 1's gate and then exits before its allreduce:
    rank 0's allreduce can never finish, and the host-side wait under the
    gate's deadline reports RankLost (the reduce aborted) instead of hanging."""
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        init = f"tcp://127.0.0.1:{_free_port()}"
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_collective_worker, args=(r, 2, init, d, die_after_gate))
                 for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(90)
            if p.exitcode is None:
                p.kill()
            assert p.exitcode == 0
        r0 = (Path(d) / "r0.txt").read_text()
        r1 = (Path(d) / "r1.txt").read_text()
    if die_after_gate < 0:
        assert (r0, r1) == ("ok", "ok")
    else:
        assert r1 == "died"
        assert r0.startswith("lost") and r0.endswith("aborted=True"), r0
        assert float(r0.split()[1]) < 30.0

"""The data-parallel QLoRA step.

One process per GPU.  The quantized base is replicated, the global batch is
sharded across ranks and split into micro-batches on each, the adapter's
gradients accumulate in the store's flat f32 buffer, one allreduce sums them
over ranks (NCCL through the library's C ABI), and one fused AdamW kernel
updates every adapter on every rank identically.

What a step does, and what it does when something is not finite, follows the
reference's TrainState::advance (engine/src/state.rs:353-400): the global
gradient norm is taken in f32 over every trained parameter; a non-finite norm
skips the update (parameters and moments stay, the optimizer's step count does
not move); a clip scales every gradient by clip/norm when the norm exceeds it.
AdamW is engine/src/optimizer.rs:305-352 (defaults beta1 0.9, beta2 0.999,
eps 1e-8, weight decay 0).
"""
from __future__ import annotations

import ctypes
import math
import os
import time
from dataclasses import dataclass

import torch

from . import ops
from ._lib import TQ_DTYPE_F32, check, lib


# ------------------------------------------------------------ batch plan ---

def shard_rows(global_rows: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of this rank's rows of the global batch (equal shards)."""
    if global_rows % world != 0:
        raise ValueError(f"a global batch of {global_rows} rows does not shard over {world} ranks")
    per = global_rows // world
    return rank * per, (rank + 1) * per


def micro_batches(rows: int, micro: int) -> list[tuple[int, int]]:
    """Equal micro-batches of this rank's rows."""
    if micro <= 0 or rows % micro != 0:
        raise ValueError(f"{rows} rows do not split into micro-batches of {micro}")
    return [(i, i + micro) for i in range(0, rows, micro)]


def grad_scale(world: int, n_micro: int) -> float:
    """Each micro-batch loss is a mean over its equal-sized part, so the mean
    over the global batch is the sum of the parts over world * n_micro."""
    return 1.0 / float(world * n_micro)


# ------------------------------------------------------------- collective ---

class NcclGradReduce:
    """Sums a flat f32 buffer over ranks with the library's NCCL communicator.

    The 128-byte NCCL id is made on rank 0 and shared through the
    torch.distributed store (plumbing only); the allreduce itself is the C ABI.
    """

    def __init__(self, rank: int, world: int, store=None):
        self.rank, self.world = rank, world
        self.comm = None
        if world == 1:
            return
        if store is None:
            import torch.distributed as dist

            store = dist.distributed_c10d._get_default_store()
        idbuf = ctypes.create_string_buffer(128)
        if rank == 0:
            check(lib().tq_dp_unique_id(idbuf))
            store.set("torobi_b200/nccl_id", bytes(idbuf.raw))
        raw = store.get("torobi_b200/nccl_id")
        ctypes.memmove(idbuf, raw, 128)
        comm = ctypes.c_void_p()
        check(lib().tq_dp_comm_init(ctypes.byref(comm), idbuf, world, rank))
        self.comm = comm

    def __call__(self, buf: torch.Tensor) -> None:
        if self.world == 1:
            return
        assert buf.dtype == torch.float32 and buf.is_contiguous()
        from .ops import _launch

        _launch("allreduce", lambda: lib().tq_dp_allreduce_sum(
            self.comm, buf.data_ptr(), buf.numel(), TQ_DTYPE_F32,
            torch.cuda.current_stream().cuda_stream), nbytes=4.0 * buf.numel())

    def watch(self, timeout: float) -> None:
        """Waits on the host, at most ``timeout`` seconds, for the collectives
        launched so far on the current stream.  A peer that died after the
        step's gate leaves its allreduce unfinished for good: on NCCL's
        asynchronous error, or when the deadline passes, the communicator is
        aborted (its kernels then return) and ``RankLost`` is raised."""
        if self.world == 1 or self.comm is None:
            return
        ev = torch.cuda.Event()
        ev.record()
        code = ctypes.c_int(0)

        def error():
            check(lib().tq_dp_comm_async_error(self.comm, ctypes.byref(code)))
            # ncclInProgress (7) is a non-blocking communicator's normal state.
            return None if code.value in (0, 7) else f"NCCL async error {code.value}"

        try:
            wait_collective(ev.query, error, timeout, self.rank, "the gradient allreduce")
        except RankLost:
            self.abort()
            raise

    def close(self) -> None:
        if self.comm is not None:
            check(lib().tq_dp_comm_destroy(self.comm))
            self.comm = None

    def abort(self) -> None:
        """Frees the communicator without its peers, after ``RankLost``."""
        if self.comm is not None:
            check(lib().tq_dp_comm_abort(self.comm))
            self.comm = None


class RankLost(RuntimeError):
    """A rank did not reach a step's collective in time (it raised, exited or
    stalled); raised on the host before any collective of that step is
    launched, so no rank is left waiting inside NCCL."""


def wait_collective(done, error, timeout: float, rank: int, what: str) -> None:
    """Polls ``done()`` until it is true; raises ``RankLost`` when ``error()``
    returns a message or ``timeout`` seconds pass first."""
    deadline = time.monotonic() + timeout
    pause = 0.0002
    while True:
        finished = done()
        # Checked after completion too: a collective can end in an error.
        msg = error()
        if msg:
            raise RankLost(f"rank {rank}: {what} failed ({msg}); a peer is gone")
        if finished:
            return
        if time.monotonic() > deadline:
            raise RankLost(f"rank {rank}: {what} did not finish within {timeout:g} s; "
                           f"a peer is gone")
        time.sleep(pause)
        pause = min(pause * 2, 0.01)


class StepGate:
    """Host-side liveness check around each step's collectives.

    Before: every rank checks in under the step's key of the torch.distributed
    store (one ``add``) and waits, polling, until all ``world`` ranks have; a
    rank that has not arrived within ``timeout`` seconds is reported as lost
    with ``RankLost``, before any collective of the step is launched.  After:
    a trainer with a gate waits for the step's allreduce on the host under the
    same deadline (``NcclGradReduce.watch``), so a peer that dies between the
    gate and the collective is reported too, with the communicator aborted.
    The reference has one process and nothing like this (its runtime poisons
    itself on a panic, engine/src/runtime.rs:105-117); it is the data-parallel
    form of "a failed step does not hang the next one".

    Keys carry a generation: the gates of one attempt of a run (one per rank)
    take the next generation from a join counter in the store, so a run that
    is restarted or restored in the same store never counts arrivals left by
    the attempt before it.  A step's key is deleted once the next step's gate
    has passed (every rank is then past it).
    """

    def __init__(self, store, rank: int, world: int, timeout: float = 240.0,
                 prefix: str = "torobi_b200/step"):
        if timeout <= 0:
            raise ValueError(f"timeout must be positive, got {timeout}")
        self.store, self.rank, self.world = store, rank, world
        self.timeout = float(timeout)
        self.generation = (store.add(f"{prefix}/joined", 1) - 1) // world if world > 1 else 0
        self.prefix = f"{prefix}/g{self.generation}"

    def key(self, step: int) -> str:
        return f"{self.prefix}/{step}"

    def wait(self, step: int) -> None:
        if self.world == 1:
            return
        key = self.key(step)
        arrived = self.store.add(key, 1)
        deadline = time.monotonic() + self.timeout
        pause = 0.0005
        while arrived < self.world:
            if time.monotonic() > deadline:
                raise RankLost(f"rank {self.rank}: {self.world - arrived} of {self.world} ranks "
                               f"did not reach step {step} within {self.timeout:g} s")
            time.sleep(pause)
            pause = min(pause * 2, 0.05)
            arrived = self.store.add(key, 0)
        if self.rank == 0 and step > 0:
            try:
                self.store.delete_key(self.key(step - 1))
            except Exception:  # noqa: BLE001  (a store without deletion keeps the key)
                pass


@dataclass
class AdamWConfig:
    lr: float = 1e-4
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    weight_decay: float = 0.0
    clip: float | None = None


class Trainer:
    """Runs QLoRA steps of a ``QLoRACausalLM`` on this rank's shard."""

    def __init__(self, model, opt: AdamWConfig | None = None, micro_batch: int = 1,
                 reduce: NcclGradReduce | None = None, rank: int = 0, world: int = 1,
                 graph: bool = False, gate: StepGate | None = None):
        self.model = model
        # gate (several ranks): checked on the host before each step's
        # allreduce, so a lost rank raises RankLost instead of hanging NCCL.
        self.gate = gate
        # graph=True replays the forward and backward of every micro-batch as
        # one CUDA graph (captured on the first step of a batch shape); the
        # collective and the optimizer stay outside it (AdamW takes the step
        # count from the host).  For small models, whose step the host's
        # per-launch work would otherwise bound.
        self.graph = graph
        self._graphs: dict[tuple, tuple] = {}
        self.opt = opt or AdamWConfig()
        self.micro = micro_batch
        self.rank, self.world = rank, world
        self.reduce = reduce or NcclGradReduce(rank, world)
        self.store = model.store
        self.norm_sq = torch.zeros(1, dtype=torch.float32, device=model.device)
        self.loss_buf = torch.zeros(1, dtype=torch.float32, device=model.device)
        self.t = 0          # AdamW step count (moves only when a step is taken)
        self.steps = 0      # steps attempted
        self.last_norm = float("nan")
        self._pending: list[float] = []  # grad scales of launched, unsettled steps

    def _gradients(self, ids: torch.Tensor) -> None:
        """Zeroes the gradient and loss buffers, then accumulates every
        micro-batch's loss and adapter gradients into them."""
        self.store.zero_grad()
        self.loss_buf.zero_()
        for a, b in micro_batches(ids.shape[0], self.micro):
            loss = self.model.loss(ids[a:b])
            loss.backward()
            self.loss_buf += loss.detach()

    def _graphed(self, ids: torch.Tensor):
        key = (tuple(ids.shape), ids.dtype)
        hit = self._graphs.get(key)
        if hit is None:
            static = ids.clone()
            # Warm up on a side stream first (first-call set-up, allocator
            # pools), as capture requires, then capture one pass.
            side = torch.cuda.Stream(device=ids.device)
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(2):
                    self._gradients(static)
            torch.cuda.current_stream().wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                self._gradients(static)
            hit = (g, static)
            self._graphs[key] = hit
        return hit

    def step(self, ids: torch.Tensor) -> torch.Tensor:
        """One optimizer step over this rank's rows ``ids`` [rows, seq] (on
        the device).  Returns the global mean loss as a device tensor."""
        st = self.store
        parts = micro_batches(ids.shape[0], self.micro)
        if self.graph:
            g, static = self._graphed(ids)
            static.copy_(ids)
            g.replay()
        else:
            self._gradients(ids)
        if self.gate is not None:
            try:
                self.gate.wait(self.steps)
            except RankLost:
                abort = getattr(self.reduce, "abort", None)
                if abort is not None:
                    abort()  # the communicator's peers are gone: do not wait on them
                raise
        self.reduce(st.grads)
        self.reduce(self.loss_buf)
        if self.gate is not None:
            watch = getattr(self.reduce, "watch", None)
            if watch is not None:
                watch(self.gate.timeout)  # RankLost (communicator aborted) if a peer died
        self.loss_buf /= float(self.world * len(parts))
        ops.sumsq(st.grads, self.norm_sq)
        o = self.opt
        gs = grad_scale(self.world, len(parts))
        # The count is advanced when the step is launched and taken back in
        # settle() if the norm turns out not finite (the kernel then moved
        # nothing), so steps can be queued without a host sync in between.
        self.t += 1
        ops.adamw_(st.params, st.grads, st.m, st.v, self.t, o.lr, o.beta1, o.beta2, o.eps,
                   o.weight_decay, grad_scale=gs, norm_sq=self.norm_sq, clip=o.clip,
                   params_bf16=st.params16)
        st.refresh_bf16()
        self.steps += 1
        self._pending.append(gs)
        return self.loss_buf

    def settle(self) -> float:
        """Reads the last step's gradient norm (a host sync).  A non-finite norm
        means the kernel skipped the update, so the AdamW count is taken back.
        Call after every step when steps may be non-finite; returns the norm of
        the averaged gradient."""
        if self._pending:
            gs = self._pending[-1]
            ns = float(self.norm_sq.item())
            if math.isfinite(ns):
                self.last_norm = math.sqrt(ns) * gs
            else:
                self.t -= 1
                self.last_norm = float("nan")
            self._pending.clear()
        return self.last_norm


def dist_env() -> tuple[int, int, int]:
    """(rank, world, local_rank) from the torchrun environment."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local

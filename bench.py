#!/usr/bin/env python
"""QLoRA training throughput on B200: tokens/s of the data-parallel step.

Workload (default): a Llama-3-8B-shaped causal LM (32 layers, hidden 4096,
32/8 heads of 128, SwiGLU 14336, vocab 128256, RoPE theta 5e5), random init,
every block linear quantized 4-bit group 64, LoRA rank 16 alpha 32 on all
seven projections, bf16 activations, f32 cross-entropy, AdamW on the adapter.
Global batch 32 x 2048 uniform random token ids, sharded over the ranks
(strong scaling: the global batch is fixed), micro-batches of 8 sequences.

    python bench.py [--gpus N --steps K --warmup W]          # this package
    python bench.py --impl reference [...]                    # the CPU port

One JSON line on rank 0.  ``value``: tokens/s over the K timed steps with the
token ids already on the device; ``e2e``: the same through the public API with
the ids copied from pinned host memory and the loss read back every step.
``roofline``: the quantized GEMM (the dominant kernel) timed live with CUDA
events around each launch on its stream, against the measured sustained bf16
tensor peak.  ``cpu_baseline``: the CPU oracle on a bounded sample.

Kernel workloads (one GPU): ``--workload qmm`` (one quantized_matmul shape),
``qmm-sweep`` (M x projection shapes, forward and dX), ``quant-sweep``
(quantize/dequantize over every Qwen2.5-0.5B-shaped linear), ``lora`` (the
LoRA down-projections and adapter gradients of one Llama-3-8B-shaped layer
and micro-batch), ``merge`` (the export merge over a Llama-3-8B-shaped layer)
and ``load`` (quantize-at-load of a published bf16 file).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "QLoRA train tokens/s at 1/2/4/8 B200; int4 qmatmul TFLOP/s and % of roofline"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# DRAM bytes (read + write) per quantized-GEMM launch of the step, from one
# ncu capture of the 2-layer step at the default micro-batch of 8 sequences
# (dram__bytes_read.sum + dram__bytes_write.sum per launch: forward 451.3 MB,
# dX 636.9 MB on average -- the dX launches of the members after the first of
# q/k/v and gate/up add into their output in the epilogue, reading it back),
# weighted to the 32-layer step's launch mix (896 forward, 884 dX launches).
# A constant: it is only as current as the kernel and micro-batch it was
# captured on.
QMM_TRAFFIC_PER_LAUNCH = {"llama3-8b": 543.5e6}


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=6)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--workload", choices=("llama3-8b", "qwen2.5-0.5b", "qmm", "qmm-sweep",
                                          "quant-sweep", "lora", "merge", "load", "attn"),
                   default="llama3-8b")
    p.add_argument("--m", type=int, default=16384, help="qmm: tokens")
    p.add_argument("--n", type=int, default=4096, help="qmm: weight rows (out features)")
    p.add_argument("--k", type=int, default=4096, help="qmm: weight cols (in features)")
    p.add_argument("--direction", choices=("fwd", "dx"), default="fwd")
    p.add_argument("--bits", type=int, choices=(4, 8), default=None,
                   help="qmm: code width (default 4); quant-sweep: only this width")
    p.add_argument("--group", type=int, choices=(32, 64, 128), default=None,
                   help="quant-sweep: only this group size")
    p.add_argument("--global-batch", type=int, default=None)
    p.add_argument("--seq", type=int, default=None)
    p.add_argument("--micro-batch", type=int, default=None)
    p.add_argument("--layers", type=int, default=None,
                   help="override the layer count (profiling runs only)")
    p.add_argument("--graph", choices=("auto", "on", "off"), default="auto",
                   help="replay each step's forward/backward as a CUDA graph "
                        "(auto: on for the launch-bound qwen2.5-0.5b step)")
    p.add_argument("--attention", choices=("native", "library"), default="library",
                   help="step workloads: this package's attention kernels or PyTorch SDPA")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def workload(args):
    import dataclasses

    from torobi_b200.model import PRESETS

    cfg = PRESETS[args.workload]
    if args.layers:
        cfg = dataclasses.replace(cfg, layers=args.layers)
    if args.workload == "llama3-8b":
        # Micro-batches of 8 sequences (16384 tokens a GEMM): 2.3 % more
        # tokens/s than 4 on one box, at a peak well inside HBM (16 gave 1 %
        # more again but peaked at 162 GB).
        gb, seq, mb = 32, 2048, 8
    else:
        gb, seq, mb = 8, 512, 8
    return cfg, args.global_batch or gb, args.seq or seq, args.micro_batch or mb


def measured_peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        try:
            return json.loads(f.read_text()), "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


# ----------------------------------------------------------- clocks ------

class ClockSampler:
    """nvidia-smi sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock samples"]}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None

        sm = sorted(x for x in (num(r[1]) for r in rows) if x is not None)
        mx = max((x for x in (num(r[2]) for r in rows) if x is not None), default=None)
        power = [x for x in (num(r[3]) for r in rows) if x is not None]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = [n for i, n in enumerate(names) if any(r[5 + i].lower() == "active" for r in rows)]
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max(power) if power else None}


# ------------------------------------------------------- CPU baseline -----

CPU_SAMPLE_TOKENS = 16


class CpuStepSample:
    """A bounded sample of the QLoRA step on the host cores: ``tokens``
    consecutive tokens (one short sequence) through one whole decoder block
    forward and backward (norms, the seven adapted quantized linears, RoPE,
    causal GQA attention, SwiGLU, the residual adds), the final norm, the
    vocabulary head and the f32 cross-entropy with their VJPs, and AdamW over
    the block's adapters -- the CPU restatement in ``oracle.decoder`` (numpy
    f32 on bf16 values, the quantized GEMMs in the C oracle)."""

    def __init__(self, cfg, tokens: int = CPU_SAMPLE_TOKENS):
        import numpy as np

        from oracle import decoder as D
        from oracle import oracle as O

        # torchrun sets OMP_NUM_THREADS=1 per rank; the baseline uses every core.
        O.set_threads(os.cpu_count() or 1)
        self.D, self.O, self.cfg, self.tokens = D, O, cfg, tokens
        self.shape = D.Shape(cfg.hidden, cfg.intermediate, cfg.heads, cfg.kv_heads,
                             cfg.head_dim, cfg.vocab, cfg.rope_theta, cfg.rms_eps, cfg.bits,
                             cfg.group, cfg.lora_rank, cfg.lora_alpha, cfg.lora_targets)
        rng = np.random.default_rng(7)
        self.blk = D.make_block(self.shape, rng)
        bound = np.float32(np.sqrt(6.0 / cfg.hidden))
        head = (rng.random((cfg.vocab, cfg.hidden), dtype=np.float32) * 2 - 1) * bound
        self.head = D.rb(head)
        del head
        self.final_norm = np.ones(cfg.hidden, np.float32)
        self.x = D.rb(rng.standard_normal((tokens, cfg.hidden), dtype=np.float32) * 0.02)
        self.targets = rng.integers(0, cfg.vocab, tokens)
        self.t = 0

    def run(self) -> dict:
        """One sample iteration; wall seconds of each part."""
        D, sh = self.D, self.shape
        parts = {"head_s": 0.0}

        def dout(out):
            t0 = time.perf_counter()
            h, rstd = D.rms_norm(out, self.final_norm, sh.rms_eps)
            self.loss, dh = D.head_loss_step(h, self.head, self.targets)
            d = D.rms_norm_vjp(out, self.final_norm, rstd, dh)
            parts["head_s"] += time.perf_counter() - t0
            return d

        t0 = time.perf_counter()
        D.block_step(sh, self.blk, self.x, dout)
        t1 = time.perf_counter()
        self.t += 1
        D.adamw_block(self.blk, self.t)
        t2 = time.perf_counter()
        parts["adamw_s"] = t2 - t1
        parts["block_s"] = (t1 - t0) - parts["head_s"]
        parts["wall_s"] = t2 - t0
        return parts

    def extrapolate(self, parts: dict, step_tokens: int) -> float:
        """Seconds of a whole step of ``step_tokens`` tokens: every layer's
        block and the head once per token, AdamW once per layer per step."""
        cfg = self.cfg
        per_tok = (cfg.layers * parts["block_s"] + parts["head_s"]) / self.tokens
        return step_tokens * per_tok + cfg.layers * parts["adamw_s"]

    def sample_text(self, parts: dict) -> str:
        return (f"{self.tokens} tokens (one sequence) through one whole decoder block forward "
                f"and backward (norms, 7 adapted 4-bit linears, RoPE, causal GQA attention over "
                f"the sample, SwiGLU), final norm, {self.cfg.vocab}-wide head and f32 "
                f"cross-entropy with VJPs, and AdamW over the block's adapters, on the CPU "
                f"restatement: block {parts['block_s']:.3f} s, head+loss {parts['head_s']:.3f} "
                f"s, AdamW {parts['adamw_s']:.4f} s per iteration; tokens/s extrapolated to "
                f"{self.cfg.layers} layers and the step's token count")

    @property
    def cores(self) -> int:
        return self.O.num_threads()


def cpu_baseline_line(cfg, step_tokens: int, iters: int, warmup: int):
    """(tokens/s extrapolated to the step, wall ms per iteration, sample
    object, parts of the best iteration)."""
    smp = CpuStepSample(cfg)
    runs = []
    for i in range(warmup + iters):
        r = smp.run()
        if i >= warmup:
            runs.append(r)
    best = min(runs, key=lambda r: r["wall_s"])
    step_s = smp.extrapolate(best, step_tokens)
    wall_ms = 1000.0 * sum(r["wall_s"] for r in runs) / len(runs)
    return step_tokens / step_s, wall_ms, smp, best


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cfg, gb, seq, mb = workload(args)
    step_tokens = gb * seq
    v, wall_ms, smp, best = cpu_baseline_line(cfg, step_tokens, args.steps, args.warmup)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        # The measured wall time of one timed iteration (the sample actually
        # run); the whole step it stands for is under extrapolated_step_s.
        "ms_per_step": wall_ms, "higher_is_better": True,
        "extrapolated_step_s": step_tokens / v,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{args.workload} QLoRA train step (CPU restatement)",
                   "global_batch": gb, "seq_len": seq, "layers": cfg.layers},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": smp.cores, "kind": "port",
                         "sample": smp.sample_text(best)},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


# -------------------------------------------------------------- ours -------

def run_ours(args):
    import torch

    from torobi_b200 import ops
    from torobi_b200.model import QLoRACausalLM
    from torobi_b200.train import AdamWConfig, NcclGradReduce, Trainer, dist_env, shard_rows

    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE is {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    cfg, gb, seq, mb = workload(args)
    lo, hi = shard_rows(gb, world, rank)
    rows = hi - lo
    if rows % mb:
        mb = rows
    model = QLoRACausalLM(cfg, dev, seed=1234, attention=args.attention)
    store = dist.distributed_c10d._get_default_store() if dist else None
    reduce = NcclGradReduce(rank, world, store)
    graph = args.graph == "on" or (args.graph == "auto" and args.workload == "qwen2.5-0.5b")
    trainer = Trainer(model, AdamWConfig(lr=1e-4), micro_batch=mb, reduce=reduce, rank=rank,
                      world=world, graph=graph)
    K, W = args.steps, args.warmup
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)
    ids_dev = torch.randint(0, cfg.vocab, (W + K, rows, seq), generator=gen, device=dev)

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(W):
        trainer.step(ids_dev[i])
        trainer.settle()
    barrier()

    clocks = ClockSampler(local)
    clocks.start()
    rec = ops.LaunchRecorder(timed=("qmm", "allreduce"))
    ops.set_recorder(rec)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(K):
        trainer.step(ids_dev[W + i])
    ev1.record()
    torch.cuda.synchronize()
    ops.set_recorder(None)
    clk = clocks.stop()
    local_ms = ev0.elapsed_time(ev1)
    ms = max_over_ranks(local_ms)
    loss = float(trainer.loss_buf.item())
    trainer.settle()
    tokens_per_step = gb * seq
    value = tokens_per_step * K / (ms / 1000.0)
    summ = rec.summary().get("qmm", {"launches": 0, "ms": 0.0, "flops": 0.0, "bytes": 0.0})
    ar = rec.summary().get("allreduce", {"launches": 0, "ms": 0.0, "bytes": 0.0})
    # NCCL's allreduce kernel is a library kernel: not counted as this package's.
    launches = rec.launches() - rec.counts.get("allreduce", 0)
    step_ms_for_share = local_ms
    roofline_timing = "every launch of the timed steps, CUDA events on its stream"
    if graph:
        # The timed steps replay a CUDA graph, whose launches no event can
        # bracket one by one: time the kernel over one eager step of the same
        # shape straight after, and count launches from it.
        trainer.graph = False
        rec = ops.LaunchRecorder(timed=("qmm",))
        ops.set_recorder(rec)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        trainer.step(ids_dev[W])
        e1.record()
        torch.cuda.synchronize()
        ops.set_recorder(None)
        trainer.settle()
        trainer.graph = True
        summ = rec.summary().get("qmm", {"launches": 0, "ms": 0.0, "flops": 0.0, "bytes": 0.0})
        launches = rec.launches() * K
        step_ms_for_share = e0.elapsed_time(e1)
        roofline_timing = ("every launch of one eager step after the timed region (the timed "
                           "steps replay a CUDA graph)")

    e2e = None
    if not args.no_e2e:
        gen_h = torch.Generator()
        gen_h.manual_seed(2000 + rank)
        ids_host = torch.randint(0, cfg.vocab, (K, rows, seq), generator=gen_h).pin_memory()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(K):
            ids = ids_host[i].to(dev, non_blocking=True)
            trainer.step(ids)
            trainer.settle()                      # gradient norm read back (the step's outcome)
            _ = float(trainer.loss_buf.item())    # loss read back
        e1.record()
        torch.cuda.synchronize()
        ms_e2e = max_over_ranks(e0.elapsed_time(e1))
        e2e = {"value": tokens_per_step * K / (ms_e2e / 1000.0), "unit": "tokens/s",
               "h2d_bytes_per_step": rows * seq * ids_host.element_size() * world,
               "d2h_bytes_per_step": 8 * world}

    ar_alone_ms = None
    grads_n = model.store.grads.numel()
    if world > 1:
        # Every rank takes these collective steps, in the same order.
        for i in range(4):
            barrier()
            a0 = torch.cuda.Event(enable_timing=True)
            a1 = torch.cuda.Event(enable_timing=True)
            a0.record()
            reduce(model.store.grads)
            a1.record()
            torch.cuda.synchronize()
            if i > 0:
                t = a0.elapsed_time(a1)
                ar_alone_ms = t if ar_alone_ms is None else min(ar_alone_ms, t)
        ar_alone_ms = max_over_ranks(ar_alone_ms)

    peaks, peak_kind = measured_peaks()
    achieved = summ["flops"] / (summ["ms"] / 1000.0) / 1e12 if summ["ms"] > 0 else 0.0
    peak = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    roofline = {
        "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
        "frac": achieved / peak if peak else None,
        "traffic": QMM_TRAFFIC_PER_LAUNCH.get(args.workload) if not args.layers else None,
        "traffic_unit": "bytes per launch (ncu, DRAM read + write)",
        "algorithmic_bytes_per_launch": summ.get("bytes", 0.0) / max(1, summ["launches"]),
        "kernel": "qmm_kernel (tcgen05 quantized_matmul, forward and dX, fused LoRA)",
        "peak_kind": f"{peak_kind} sustained bf16 (cuBLAS, long loop)",
        "launches_timed": int(summ["launches"]),
        "share_of_step": summ["ms"] / max(1e-9, step_ms_for_share),
        "timing": roofline_timing,
    }

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tps, _, smp, best = cpu_baseline_line(cfg, tokens_per_step, 2, 1)
        cpu = {"value": tps, "unit": "tokens/s", "cores": smp.cores, "kind": "port",
               "sample": smp.sample_text(best)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (uniform random token ids, random-init weights)",
            "config": {"workload": f"{args.workload} QLoRA train step", "global_batch": gb,
                       "seq_len": seq, "micro_batch": mb, "parallelism": f"dp{world}",
                       "cuda_graph": graph, "attention": args.attention,
                       "layers": cfg.layers, "quant": f"{cfg.bits}-bit g{cfg.group}",
                       "lora": f"r{cfg.lora_rank} a{int(cfg.lora_alpha)} on "
                               f"{'+'.join(cfg.lora_targets)}",
                       "l2": "inputs larger than L2 (quantized base weights "
                             f"{model.base_nbytes() / 1e9:.2f} GB read per step)"},
            "model_tflops_per_s": value * cfg.flops_per_token(seq) / 1e12,
            "loss": loss,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clk,
        }
        if world > 1:
            # The gradient (and loss) allreduce, CUDA events around each NCCL
            # call on rank 0's stream inside the timed steps (includes any wait
            # for a slower rank), and the gradient allreduce alone after a
            # barrier (the collective's own time).
            line["allreduce"] = {"ms_per_step": ar["ms"] / K, "launches_per_step":
                                 ar["launches"] / K, "bytes_per_step": ar["bytes"] / K,
                                 "share_of_step": ar["ms"] / local_ms if local_ms else None,
                                 "isolated_ms": ar_alone_ms,
                                 "isolated_bus_gbs": (2.0 * (world - 1) / world * 4.0 *
                                                      grads_n / ar_alone_ms / 1e6)}
        print(json.dumps(line), flush=True)
    reduce.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------ kernel workloads ---

# quantized_matmul shapes: Llama-3-8B projections (4096x4096, 1024x4096,
# 14336x4096, 4096x14336) and Llama-3-70B ones (8192x8192, 28672x8192,
# 8192x28672), as (w_rows = out features, w_cols = in features).
QMM_SHAPES = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (8192, 8192),
              (28672, 8192), (8192, 28672)]
QMM_MS = [16, 128, 1024, 4096, 16384]


def _time_kernel(fn, iters, warmup, flush):
    """Mean CUDA-event time of fn() with an L2 flush before every launch;
    the flush runs outside the timed events."""
    import torch

    for _ in range(warmup):
        flush()
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        flush()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        total += s.elapsed_time(e)
    return total / iters


def _qmm_case(m, n, k, direction, dev, seed=0, bits=4):
    import torch

    from torobi_b200 import ops

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    w = (torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16()
    c, s, b = ops.quantize(w, 64, bits)
    del w
    if direction == "fwd":
        x = torch.randn(m, k, device=dev, generator=g).bfloat16()
        return (lambda: ops.quantized_matmul(x, c, s, b, True, 64, bits)), (x, c, s, b)
    dy = torch.randn(m, n, device=dev, generator=g).bfloat16()
    return (lambda: ops.quantized_matmul(dy, c, s, b, False, 64, bits)), (dy, c, s, b)


def _grouped_quant_ms(stacks, layers, grp, bits, K, W, flush):
    """CUDA-event ms of one tq_quantize_batch and one tq_dequantize_batch over
    every layer's matrix of every stacked shape (len(stacks) * layers jobs)."""
    import torch

    from torobi_b200._lib import TqDequantizeJob, TqQuantizeJob, lib

    mats = [st[l * (st.shape[0] // layers):(l + 1) * (st.shape[0] // layers)]
            for st in stacks for l in range(layers)]
    n = len(mats)
    qjobs, djobs = (TqQuantizeJob * n)(), (TqDequantizeJob * n)()
    keep = []
    for i, w in enumerate(mats):
        r, c = w.shape
        codes = torch.empty(r, c * bits // 32, dtype=torch.uint32, device=w.device)
        sc = torch.empty(r, c // grp, dtype=torch.bfloat16, device=w.device)
        bi = torch.empty_like(sc)
        out = torch.empty_like(w)
        keep += [codes, sc, bi, out]
        qjobs[i] = TqQuantizeJob(w.data_ptr(), r, c, codes.data_ptr(), sc.data_ptr(), bi.data_ptr())
        djobs[i] = TqDequantizeJob(codes.data_ptr(), sc.data_ptr(), bi.data_ptr(), r, c,
                                   out.data_ptr())
    L = lib()
    stream = torch.cuda.current_stream().cuda_stream

    def q():
        assert L.tq_quantize_batch(qjobs, n, grp, bits, stream) == 0

    def dq():
        assert L.tq_dequantize_batch(djobs, n, grp, bits, stream) == 0

    gq = _time_kernel(q, K, W, flush)
    gdq = _time_kernel(dq, K, W, flush)
    del keep
    return gq, gdq


def run_kernels(args):
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    # Write 1 GiB (> 126 MB of L2), then read another 1 GiB, so that L2 is
    # left holding clean lines: a kernel timed after a write-only flush also
    # pays for writing back the flush's dirty lines it evicts (up to 126 MB),
    # which halves the apparent rate of an HBM-bound kernel of ~100 MB.  Long
    # enough that the host has enqueued the timed launch before the flush
    # ends, so the events time the device only.
    flush_buf = torch.empty(1024 * 1024 * 1024, dtype=torch.uint8, device=dev)
    flush_src = torch.ones(256 * 1024 * 1024, dtype=torch.int32, device=dev)

    def flush():
        flush_buf.zero_()
        flush_src.max()
    peaks, peak_kind = measured_peaks()
    burst = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    K, W = args.steps, args.warmup
    common = {"n_gpus": 1, "steps": K, "warmup": W, "higher_is_better": True,
              "vs_baseline": None, "data": "synthetic"}
    if args.workload == "qmm":
        bits = args.bits or 4
        fn, _ = _qmm_case(args.m, args.n, args.k, args.direction, dev, bits=bits)
        ms = _time_kernel(fn, K, W, flush)
        tf = 2.0 * args.m * args.n * args.k / (ms / 1000.0) / 1e12
        print(json.dumps({"metric": "int4 quantized_matmul TFLOP/s", "value": tf,
                          "unit": "TFLOP/s", "ms_per_step": ms, "scaling": "weak",
                          "dtype": "bf16", **common,
                          "config": {"workload": f"quantized_matmul {args.direction}",
                                     "m": args.m, "w_rows": args.n, "w_cols": args.k,
                                     "bits": bits, "group_size": 64,
                                     "l2": "flushed before every launch (clean)"},
                          "roofline": {"bound": "tensor", "achieved": tf, "peak": burst,
                                       "unit": "TFLOP/s", "frac": tf / burst,
                                       "peak_kind": f"{peak_kind} burst bf16"}}), flush=True)
        return 0
    if args.workload == "qmm-sweep":
        rows = []
        for n, k in QMM_SHAPES:
            for m in QMM_MS:
                for d in ("fwd", "dx"):
                    fn, keep = _qmm_case(m, n, k, d, dev)
                    ms = _time_kernel(fn, K, W, flush)
                    fl = 2.0 * m * n * k
                    byts = m * k * 2 + n * k * (0.5 + 4 / 64) + m * n * 2
                    tf = fl / (ms / 1000.0) / 1e12
                    gbs = byts / (ms / 1000.0) / 1e9
                    bound = "hbm" if fl / byts < burst * 1e12 / (hbm * 1e9) else "tensor"
                    frac = gbs / hbm if bound == "hbm" else tf / burst
                    rows.append({"m": m, "w_rows": n, "w_cols": k, "dir": d, "ms": ms,
                                 "tflops": tf, "gbs": gbs, "bound": bound, "frac": frac})
                    print(json.dumps(rows[-1]), file=sys.stderr, flush=True)
                    del keep, fn
        big = [r["tflops"] for r in rows if r["m"] >= 4096]
        val = sum(big) / len(big)
        print(json.dumps({"metric": "int4 quantized_matmul TFLOP/s (mean over M>=4096)",
                          "value": val, "unit": "TFLOP/s", "scaling": "weak", "dtype": "bf16",
                          **common,
                          "config": {"workload": "quantized_matmul shape sweep, 4-bit g64",
                                     "l2": "flushed before every launch (clean)"},
                          "roofline": {"bound": "tensor", "achieved": val, "peak": burst,
                                       "unit": "TFLOP/s", "frac": val / burst,
                                       "peak_kind": f"{peak_kind} burst bf16"},
                          "sweep": rows}), flush=True)
        return 0
    if args.workload == "quant-sweep":
        from torobi_b200 import ops
        from torobi_b200.model import QWEN2_5_0_5B

        shapes = list(QWEN2_5_0_5B.linear_shapes().values())
        g = torch.Generator(device=dev)
        g.manual_seed(0)
        mats = [(torch.randn(o, i, device=dev, generator=g) * 0.02).bfloat16() for o, i in shapes]
        for wm in mats:
            mask = torch.rand(wm.shape, device=dev, generator=g) < 0.001
            sign = torch.where(torch.rand(wm.shape, device=dev, generator=g) < 0.5, -0.5, 0.5)
            wm[mask] = sign[mask].bfloat16()
        # Each shape stacked over the 24 layers, so a launch is HBM-sized.
        big = [torch.cat([wm] * QWEN2_5_0_5B.layers) for wm in mats]
        rows = []
        for bits in (4, 8) if args.bits is None else (args.bits,):
            for grp in (32, 64, 128) if args.group is None else (args.group,):
                tq_ms = tdq_ms = 0.0
                nbytes = 0.0
                for wm in big:
                    tq_ms += _time_kernel(lambda: ops.quantize(wm, grp, bits), K, W, flush)
                    c, s_, b_ = ops.quantize(wm, grp, bits)
                    tdq_ms += _time_kernel(lambda: ops.dequantize(c, s_, b_, grp, bits), K, W,
                                           flush)
                    nbytes += wm.numel() * (2 + bits / 8 + 4 / grp)
                # The same bytes as one grouped launch over the 168 matrices
                # (each shape's 24 layers as separate [rows, cols] views), the
                # job tables built before the timed region.
                gq_ms, gdq_ms = _grouped_quant_ms(big, QWEN2_5_0_5B.layers, grp, bits, K, W,
                                                  flush)
                rows.append({"bits": bits, "group": grp, "quantize_gbs": nbytes / tq_ms / 1e6,
                             "dequantize_gbs": nbytes / tdq_ms / 1e6,
                             "grouped_quantize_gbs": nbytes / gq_ms / 1e6,
                             "grouped_dequantize_gbs": nbytes / gdq_ms / 1e6, "bytes": nbytes})
                print(json.dumps(rows[-1]), file=sys.stderr, flush=True)
        val = sum(r["dequantize_gbs"] for r in rows) / len(rows)
        print(json.dumps({"metric": "quantize/dequantize GB/s (Qwen2.5-0.5B shapes, 24 layers)",
                          "value": val, "unit": "GB/s", "scaling": "weak",
                          "dtype": "u4/u8 codes, bf16", **common,
                          "config": {"workload": "affine quantize/dequantize sweep",
                                     "l2": "flushed before every launch (clean)"},
                          "roofline": {"bound": "hbm", "achieved": val, "peak": hbm,
                                       "unit": "GB/s", "frac": val / hbm,
                                       "peak_kind": f"{peak_kind} copy"},
                          "sweep": rows}), flush=True)
        return 0
    if args.workload == "lora":
        # The skinny LoRA launches of one Llama-3-8B-shaped layer for one
        # micro-batch of 8192 tokens (rank 16): per linear [d_out, d_in], the
        # forward down-projection x.A^T (reads x [8192, d_in]), the backward
        # one dY.B (reads dY [8192, d_out]) and the two adapter gradients
        # (dA reads x, dB reads dY).  HBM-bound on the big operand.
        from torobi_b200 import ops
        from torobi_b200.model import LLAMA3_8B

        g = torch.Generator(device=dev)
        g.manual_seed(0)
        r, m = LLAMA3_8B.lora_rank, 8192
        kinds = {"down": [0.0, 0.0], "grad": [0.0, 0.0]}
        rows = []
        for name, (o, i) in LLAMA3_8B.linear_shapes().items():
            for side, c in (("x", i), ("dY", o)):
                big = torch.randn(m, c, device=dev, generator=g).bfloat16()
                a = (torch.randn(r, c, device=dev, generator=g) * 0.01).bfloat16()
                _, p_t = ops.lora_down(big, a, 2.0)
                ms_d = _time_kernel(lambda: ops.lora_down(big, a, 2.0), K, W, flush)
                out = torch.empty(c, r, dtype=torch.float32, device=dev)
                ms_g = _time_kernel(lambda: ops.lora_grad(big, p_t, 0, out=out), K, W, flush)
                nb_d = m * c * 2 + 2 * m * r * 2
                nb_g = m * c * 2 + r * m * 2 + c * r * 4
                kinds["down"][0] += ms_d
                kinds["down"][1] += nb_d
                kinds["grad"][0] += ms_g
                kinds["grad"][1] += nb_g
                rows.append({"linear": name, "operand": side, "m": m, "k": c,
                             "down_us": ms_d * 1e3, "down_gbs": nb_d / ms_d / 1e6,
                             "grad_us": ms_g * 1e3, "grad_gbs": nb_g / ms_g / 1e6})
                del big, a, p_t, out
        total_ms = kinds["down"][0] + kinds["grad"][0]
        val = (kinds["down"][1] + kinds["grad"][1]) / total_ms / 1e6
        print(json.dumps({"metric": "LoRA skinny kernels GB/s (Llama-3-8B layer, 8192 tokens, r16)",
                          "value": val, "unit": "GB/s", "scaling": "weak", "dtype": "bf16",
                          **common,
                          "config": {"workload": "lora_down + lora_grad over one layer",
                                     "l2": "flushed before every launch (clean)"},
                          "roofline": {"bound": "hbm", "achieved": val, "peak": hbm,
                                       "unit": "GB/s", "frac": val / hbm,
                                       "peak_kind": f"{peak_kind} copy"},
                          "down_gbs": kinds["down"][1] / kinds["down"][0] / 1e6,
                          "grad_gbs": kinds["grad"][1] / kinds["grad"][0] / 1e6,
                          "launches": rows}), flush=True)
        return 0
    if args.workload == "merge":
        # The export merge over one Llama-3-8B-shaped layer's seven linears
        # (4-bit g64, LoRA r16): reads bits/8 + 4/g bytes of packed weight
        # and writes 4 bytes of f32 per element.
        from torobi_b200 import ops
        from torobi_b200.model import LLAMA3_8B

        g = torch.Generator(device=dev)
        g.manual_seed(0)
        r = LLAMA3_8B.lora_rank
        total_ms = 0.0
        nbytes = 0.0
        rows = []
        for name, (o, i) in LLAMA3_8B.linear_shapes().items():
            c, s_, b_ = ops.quantize((torch.randn(o, i, device=dev, generator=g) * 0.02)
                                     .bfloat16(), 64, 4)
            a = torch.randn(r, i, device=dev, generator=g) * 0.01
            bb = torch.randn(o, r, device=dev, generator=g) * 0.01
            ms = _time_kernel(lambda: ops.lora_merge(c, s_, b_, 64, 4, lora_a=a, lora_b=bb,
                                                     scale=2.0), K, W, flush)
            nb = o * i * (0.5 + 4 / 64 + 4)
            rows.append({"linear": name, "rows": o, "cols": i, "ms": ms, "gbs": nb / ms / 1e6})
            total_ms += ms
            nbytes += nb
        val = nbytes / total_ms / 1e6
        print(json.dumps({"metric": "LoRA merge for export GB/s (Llama-3-8B layer, r16)",
                          "value": val, "unit": "GB/s", "scaling": "weak", "dtype": "u4 -> f32",
                          **common,
                          "config": {"workload": "dequantize + scale * B A, f32 out",
                                     "l2": "flushed before every launch (clean)"},
                          "roofline": {"bound": "hbm", "achieved": val, "peak": hbm,
                                       "unit": "GB/s", "frac": val / hbm,
                                       "peak_kind": f"{peak_kind} copy"},
                          "linears": rows}), flush=True)
        return 0
    if args.workload == "attn":
        # Causal grouped-query attention at the two models' head shapes, this
        # package's tensor-core kernels against the library SDPA (PyTorch's
        # fused attention) on the same inputs, forward and forward+backward.
        import torch.nn.functional as F

        from torobi_b200 import glue

        rows = []
        for name, (b, sq, h, hk, d) in (("llama3-8b", (4, 2048, 32, 8, 128)),
                                         ("qwen2.5-0.5b", (8, 512, 14, 2, 64))):
            g = torch.Generator(device=dev)
            g.manual_seed(0)
            q = torch.randn(b, sq, h, d, device=dev, generator=g).bfloat16()
            k = torch.randn(b, sq, hk, d, device=dev, generator=g).bfloat16()
            v = torch.randn(b, sq, hk, d, device=dev, generator=g).bfloat16()
            # causal: sq * (sq + 1) / 2 score entries per head, two matmuls
            flops = 2.0 * 2.0 * b * h * d * sq * (sq + 1) / 2

            def ours():
                glue.attention_forward(q, k, v, True)

            def lib_sdpa():
                F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                               v.transpose(1, 2), is_causal=True,
                                               enable_gqa=h != hk)

            do = torch.randn(b, sq, h, d, device=dev, generator=g).bfloat16()
            o, lse = glue.attention_forward(q, k, v, True)
            qt, kt, vt = (t.transpose(1, 2).detach().requires_grad_() for t in (q, k, v))
            ol = F.scaled_dot_product_attention(qt, kt, vt, is_causal=True, enable_gqa=h != hk)
            dot = do.transpose(1, 2)

            def ours_bwd():
                glue.attention_backward(q, k, v, o, do, lse, True)

            def lib_bwd():
                torch.autograd.grad(ol, (qt, kt, vt), dot, retain_graph=True)

            ms_o = _time_kernel(ours, K, W, flush)
            ms_l = _time_kernel(lib_sdpa, K, W, flush)
            ms_ob = _time_kernel(ours_bwd, K, W, flush)
            ms_lb = _time_kernel(lib_bwd, K, W, flush)
            # backward: five matmuls of the forward's size (S, dP, dV, dK, dQ)
            rows.append({"shape": name, "batch": b, "seq": sq, "heads": h, "kv_heads": hk,
                         "dim": d, "fwd_ms": ms_o, "fwd_tflops": flops / ms_o / 1e9,
                         "library_fwd_ms": ms_l, "library_fwd_tflops": flops / ms_l / 1e9,
                         "bwd_ms": ms_ob, "bwd_tflops": 2.5 * flops / ms_ob / 1e9,
                         "library_bwd_ms": ms_lb, "library_bwd_tflops": 2.5 * flops / ms_lb / 1e9})
            print(json.dumps(rows[-1]), file=sys.stderr, flush=True)
        val = rows[0]["fwd_tflops"]
        peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        print(json.dumps({"metric": "causal GQA attention TFLOP/s (Llama-3-8B heads, seq 2048)",
                          "value": val, "unit": "TFLOP/s", "scaling": "weak", "dtype": "bf16",
                          **common,
                          "config": {"workload": "attention forward, 4 x 2048, 32/8 heads of 128",
                                     "l2": "flushed before every launch (clean)"},
                          "roofline": {"bound": "tensor", "achieved": val, "peak": peak,
                                       "unit": "TFLOP/s", "frac": val / peak,
                                       "peak_kind": f"{peak_kind} burst bf16"},
                          "shapes": rows}), flush=True)
        return 0
    if args.workload == "load":
        # Quantize-at-load of a published dense bf16 file (Llama-3-8B shapes,
        # --layers deep, default 2): file -> host -> device -> quantized.
        import dataclasses
        import shutil

        from torobi_b200.model import LLAMA3_8B, QLoRACausalLM
        from torobi_b200.weights import published_parameters, write_dense

        cfg = dataclasses.replace(LLAMA3_8B, layers=args.layers or 2)
        tmp = Path(tempfile.mkdtemp(prefix="tq_load_"))
        try:
            gcpu = torch.Generator().manual_seed(0)
            dense = {d.path: (torch.randn(d.shape, generator=gcpu) * 0.02).bfloat16()
                     for d in published_parameters(cfg)}
            f = tmp / "model.safetensors"
            write_dense(f, dense, metadata={"format": "pt"})
            lin = sum(t.numel() * 2 for k, t in dense.items() if k.endswith("_proj.weight"))
            total = sum(t.numel() * 2 for t in dense.values())
            del dense
            times = []
            for it in range(W + K):
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                m = QLoRACausalLM.from_pretrained(cfg, f, device=dev)
                torch.cuda.synchronize()
                if it >= W:
                    times.append(time.perf_counter() - t0)
                del m
            sec = sorted(times)[len(times) // 2]
        finally:
            shutil.rmtree(tmp, ignore_errors=True)
        print(json.dumps({"metric": "quantize-at-load GB/s (published bf16 file to a QLoRA model)",
                          "value": total / sec / 1e9, "unit": "GB/s", "scaling": "weak",
                          "dtype": "bf16 -> u4", **common, "ms_per_step": sec * 1e3,
                          "config": {"workload": "from_pretrained, Llama-3-8B shapes",
                                     "layers": cfg.layers, "file_bytes": total,
                                     "linear_bytes": lin,
                                     "linear_gbs": lin / sec / 1e9,
                                     "timing": "wall clock, file in the page cache"}}),
              flush=True)
        return 0
    raise SystemExit(f"unknown kernel workload {args.workload}")


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload in ("qmm", "qmm-sweep", "quant-sweep", "lora", "merge", "load", "attn"):
        return run_kernels(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

"""Generates the golden fixtures in this folder from the CPU oracle.

    python tests/golden/make_golden.py

quantize.npz  small bf16 matrices (seeded normal rows plus edge rows: zeros,
              constants, one-signed ramps, subnormals, NaN/inf) with their
              codes, scales, biases and dequantized values for every
              bits x group_size pair.
qlora.npz     one small adapted linear (M=48, K=192, N=136, rank 8, alpha 16,
              4-bit group 64, with a bias) with y, dx, dA, dB.

MLX (the dependency that owns these ops) cannot run here, so these pin the
oracle's stated conventions against accidental change; they are not MLX
outputs.  Re-run only when a convention is changed on purpose.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import oracle as O  # noqa: E402


def edge_rows(cols: int) -> np.ndarray:
    f = np.float32
    rows = [np.zeros(cols, f), np.full(cols, 0.75, f), np.full(cols, -3.0, f),
            -np.abs(np.linspace(0.1, 2.0, cols, dtype=f)), np.linspace(-1.0, 0.5, cols, dtype=f),
            np.linspace(-0.5, 1.0, cols, dtype=f), np.full(cols, 1e-40, f)]
    r = np.linspace(-1.0, 1.0, cols, dtype=f); r[3] = np.nan; rows.append(r)
    r = np.linspace(-1.0, 1.0, cols, dtype=f); r[5] = np.inf; rows.append(r)
    return np.stack(rows)


def main() -> None:
    rng = np.random.default_rng(20261201)
    out = {}
    for bits in (4, 8):
        for group in (32, 64, 128):
            normal = rng.standard_normal((6, 256), dtype=np.float32) * np.float32(0.02)
            w = O.bf16_from_f32(np.concatenate([normal, edge_rows(256)]))
            c, s, b = O.quantize(w, bits, group)
            tag = f"{bits}_{group}"
            out[f"w_{tag}"] = w
            out[f"codes_{tag}"] = c
            out[f"scales_{tag}"] = s
            out[f"biases_{tag}"] = b
            out[f"deq_{tag}"] = O.dequantize(c, s, b, bits, group)
    np.savez_compressed(HERE / "quantize.npz", **out)

    rng = np.random.default_rng(1)
    M, K, N, r, alpha = 48, 192, 136, 8, 16.0
    x = O.normal_bf16(rng, (M, K))
    w = O.normal_bf16(rng, (N, K), 0.02)
    a = O.normal_bf16(rng, (r, K), 1.0 / 8.0)
    bl = O.normal_bf16(rng, (N, r), 0.01)
    bias = O.normal_bf16(rng, (N,), 0.1)
    dy = O.normal_bf16(rng, (M, N))
    c, s, b = O.quantize(w, 4, 64)
    f = O.f32_from_bf16
    y, _ = O.qlora_linear_fwd(f(x), c, s, b, f(a), f(bl), alpha / r, 4, 64, bias=f(bias))
    dx, da, db = O.qlora_linear_bwd(f(x), f(dy), c, s, b, f(a), f(bl), alpha / r, 4, 64)
    np.savez_compressed(HERE / "qlora.npz", x=x, w=w, lora_a=a, lora_b=bl, bias=bias, dy=dy,
                        codes=c, scales=s, biases=b, y=O.bf16_from_f32(y),
                        dx=O.bf16_from_f32(dx), da=O.bf16_from_f32(da), db=O.bf16_from_f32(db),
                        meta=np.array([M, K, N, r, int(alpha), 4, 64]))
    print("wrote", HERE / "quantize.npz", HERE / "qlora.npz")


if __name__ == "__main__":
    main()

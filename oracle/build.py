"""Build recipe for the C oracle (test infrastructure only).

Compiles ``oracle/qlora_oracle.c`` into ``oracle/_build/`` twice: a portable
x86-64 build and an AVX-512 build.  ``oracle.oracle`` loads the AVX-512 one
only when the host CPU reports ``avx512f``.  Both are compiled with
``-ffp-contract=off`` so every f32 operation rounds exactly as written, which
the bit-exact quantize parity relies on.

The reference's own implementation of this path cannot be built here: it is
Rust (engine/) plus the prebuilt MLX 0.32.2 static libraries that
lib/torobi/mlx_prebuilt.rb downloads, and neither cargo nor MLX is present.
So there is no ``oracle/_ref``.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "qlora_oracle.c"
OUT = HERE / "_build"

VARIANTS = {
    "liboracle.so": ["-O3"],
    "liboracle_avx512.so": ["-O3", "-march=skylake-avx512", "-mprefer-vector-width=512"],
}


def _stale(target: Path) -> bool:
    return not target.exists() or target.stat().st_mtime < SRC.stat().st_mtime


def build(force: bool = False, verbose: bool = False) -> Path:
    OUT.mkdir(exist_ok=True)
    for name, flags in VARIANTS.items():
        target = OUT / name
        if not force and not _stale(target):
            continue
        tmp = OUT / (name + f".tmp{os.getpid()}")
        cmd = ["gcc", *flags, "-std=c11", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
               "-fPIC", "-shared", "-Wall", str(SRC), "-o", str(tmp), "-lm"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        os.replace(tmp, target)
    return OUT


if __name__ == "__main__":
    build(force=True, verbose=True)

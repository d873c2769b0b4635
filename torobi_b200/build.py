"""Build recipe for libtorobi_b200.so (sm_100a).

Every ``csrc/*.cu`` is compiled by nvcc for ``sm_100a`` (the arch-specific
target that carries tcgen05 and the TMA tensor copies) into ``_build/`` and
linked, with static cudart and NCCL, into ``torobi_b200/libtorobi_b200.so``.
The library is built in-tree so it travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libtorobi_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda) / "bin" / "nvcc"
    return str(path) if path.exists() else (shutil.which("nvcc") or "nvcc")


def _nccl_flags() -> list[str]:
    for inc in ("/usr/include", "/usr/local/include"):
        if Path(inc, "nccl.h").exists():
            return [f"-I{inc}"]
    return []


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) +
                  list((ROOT / "include").glob("*.h")))


def _stale(obj: Path, src: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def compile_one(src: Path, verbose: bool = False, extra: list[str] | None = None) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-Wall", "--expt-relaxed-constexpr", *_nccl_flags(),
           *(extra or []), "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = _headers()
    srcs = _sources()
    todo = [s for s in srcs if force or ptxas_v or _stale(BUILD / (s.stem + ".o"), s, headers)]
    extra = ["-Xptxas", "-v"] if ptxas_v else None
    if todo:
        with ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            list(ex.map(lambda s: compile_one(s, verbose, extra), todo))
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", *[str(o) for o in objs],
               "-o", str(tmp), "-lnccl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_v="--ptxas-v" in sys.argv)

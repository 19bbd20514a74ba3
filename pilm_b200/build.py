"""Build libpilm_cuda.so (sm_100a) from pilm_b200/csrc with nvcc, in-tree.

    python -m pilm_b200.build            # or: import pilm_b200.build; build()

The library is written next to this file so that it ships with the package and
with snapshots of the repository; it is rebuilt only when a source is newer.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libpilm_cuda.so"
INCLUDE = HERE.parent / "include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["runtime.cu", "linear.cu", "linear_tc.cu", "norm.cu", "attention.cu", "accept.cu", "mtp.cu", "f32.cu"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(INCLUDE),
                    "--expt-relaxed-constexpr"]
    if verbose:
        flags += ["-Xptxas", "-v"]
    objs = []
    for src in SOURCES:
        obj = objdir / (Path(src).stem + ".o")
        cmd = [nvcc()] + flags + ["-c", str(CSRC / src), "-o", str(obj)]
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc()] + ARCH + ["-shared", "-o", str(tmp)] + objs, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)

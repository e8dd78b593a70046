"""Build recipe for libb200gemv.so (the C-ABI library) -- sm_100a only.

    python llama-3.2-3b-instruct-gemm-optimization_b200/build.py

nvcc compiles the kernels and the host API straight into one shared library
next to this file; nothing is JIT-compiled or installed into site-packages.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libb200gemv.so"
SOURCES = ["gemv.cu", "pack.cu", "static_scratch.cu", "api.cpp"]
HEADERS = ["device.cuh", "gemv.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [HERE.parent / "include" / "b200gemv.h"]
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False, out: Path = LIB, defines=()) -> Path:
    if not force and out == LIB and not stale():
        return LIB
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "-shared",
           "-I", str(HERE.parent / "include"), *[f"-D{d}" for d in defines], "-o", str(out)] + \
        [str(CSRC / s) for s in SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return out


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)

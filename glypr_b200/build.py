"""Build libglypr_cuda.so in-tree with nvcc for sm_100a (no GPU needed to compile)."""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libglypr_cuda.so")
SOURCES = ["glypr_cuda.cu", "gguf.cpp", "engine.cpp", "tokenizer.cpp"]
HEADERS = ["common.cuh", "gemm.cuh", "q8gemm.cuh", "attention_tc.cuh", "attention_d512.cuh", "attention_pair.cuh", "rowops.cuh", "gguf.h", "unicode_case.inc"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def command(extra=()) -> list:
    return [
        nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
        "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O3", "-shared",
        "-I", os.path.join(ROOT, "include"), "-I", CSRC,
        *[os.path.join(CSRC, s) for s in SOURCES],
        "-o", LIB, "-cudart", "static", "-lpthread", "-ldl", "-lrt", *extra,
    ]


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(ROOT, "include", "glypr_cuda.h")]
    return any(os.path.getmtime(p) > t for p in deps if os.path.exists(p))


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    if force or stale():
        cmd = command(extra)
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=["-Xptxas", "-v"] if "--ptxas" in sys.argv else [])

"""Build libgemma_b200.so (sm_100a) in-tree with nvcc.

Usage: python webgpu-gemma_b200/build.py [--force] [--verbose]
The library lands next to the Python package (gemma_b200/libgemma_b200.so), so it travels
with the source tree to the GPU machine.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT = os.path.join(HERE, "gemma_b200", "libgemma_b200.so")
SOURCES = ["gg_engine.cu", "gg_step.cu", "gg_decode.cu", "gg_gemm.cu", "gg_prefill.cu", "gg_tokenizer.cpp"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr", "-I", INCLUDE]


def _deps():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    files.append(os.path.join(INCLUDE, "gemma_b200.h"))
    return files


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and os.path.exists(OUT):
        t = os.path.getmtime(OUT)
        if all(os.path.getmtime(f) <= t for f in _deps()):
            return OUT
    tmp = OUT + f".tmp{os.getpid()}"
    cmd = [NVCC, *FLAGS, "-Xptxas", "-v", *[os.path.join(CSRC, s) for s in SOURCES], "-o", tmp]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libgemma_b200.so")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)

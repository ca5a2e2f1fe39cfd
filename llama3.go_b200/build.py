"""Builds libl3g.so (sm_100a) in-tree with nvcc.

    python llama3.go_b200/build.py [--force] [--ptxas-verbose]

The library is written next to this file so that it travels with the source
tree; ``l3g.py`` loads it from there and fails loudly when it is missing.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libl3g.so")
SOURCES = [os.path.join(CSRC, f) for f in ("l3g_runtime.cu", "l3g_gguf.cpp")]


def deps():
    """Every source and header the library is built from."""
    files = [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))
             if f.endswith((".cu", ".cuh", ".cpp", ".h"))]
    return files + [os.path.join(ROOT, "include", "l3g.h"), os.path.abspath(__file__)]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(d) > t for d in deps())


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = False) -> str:
    if not force and not stale():
        return LIB
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC,-O2", "-I", os.path.join(ROOT, "include"), "-I", CSRC,
           *SOURCES, "-o", LIB + ".tmp", "-ldl"]
    if ptxas_verbose:
        cmd.insert(1, "-Xptxas=-v")
    if not quiet:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args()
    build(force=args.force, ptxas_verbose=args.ptxas_verbose)
    sys.exit(0)

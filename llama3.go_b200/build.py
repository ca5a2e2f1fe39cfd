"""Builds libl3g.so (sm_100a) in-tree with nvcc.

    python llama3.go_b200/build.py [--force] [--ptxas-verbose]

Each translation unit of the runtime is compiled to an object in parallel
(each is its own device module), then they are linked into the library.
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
UNITS = ["l3g_api.cu", "l3g_model.cu", "l3g_tp.cu", "l3g_step.cu", "l3g_persist_host.cu",
         "l3g_batched.cu", "l3g_gguf.cpp"]
OBJDIR = os.path.join(HERE, "_build")


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


def _compile(unit: str, ptxas_verbose: bool, quiet: bool) -> str:
    src = os.path.join(CSRC, unit)
    obj = os.path.join(OBJDIR, unit.rsplit(".", 1)[0] + ".o")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
           "-I", os.path.join(ROOT, "include"), "-I", CSRC, "-c", src, "-o", obj]
    if ptxas_verbose:
        cmd.insert(1, "-Xptxas=-v")
    if not quiet:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0 or (ptxas_verbose and not quiet):
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode != 0:
        raise subprocess.CalledProcessError(r.returncode, cmd)
    return obj


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = False) -> str:
    if not force and not stale():
        return LIB
    from concurrent.futures import ThreadPoolExecutor
    os.makedirs(OBJDIR, exist_ok=True)
    with ThreadPoolExecutor(max_workers=len(UNITS)) as ex:
        objs = list(ex.map(lambda u: _compile(u, ptxas_verbose, quiet), UNITS))
    cmd = [nvcc(), *ARCH, "-shared", *objs, "-o", LIB + ".tmp", "-ldl"]
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

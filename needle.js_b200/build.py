"""Builds libneedle_cuda.so in-tree with nvcc for sm_100a (B200) only.

No PyTorch is involved: the library links the CUDA runtime statically and exposes the C-ABI
declared in include/needle_cuda.h.  --fmad=false keeps every binary64/binary32 multiply and add
separately rounded, as the reference's JavaScript arithmetic is; the kernels request fused
multiply-adds explicitly (fma()) only where the product is exact.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libneedle_cuda.so")
SOURCES = ["engine.cu", "cq.cu", "layer.cu", "ops.cu", "attn_fast.cu", "cq_fast.cu", "cq_gemm_tc.cu", "grammar.cpp"]
HEADERS = ["common.cuh", "cq.cuh", "engine.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "--fmad=false", "-std=c++17", "--extended-lambda", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-Wall", "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles every source (in parallel) and links the shared library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", h)
                                                          for h in ("needle_cuda.h", "needle_grammar.h")]
    objs, jobs = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            jobs.append([nvcc(), *ARCH, *FLAGS, "-c", s, "-o", o])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
        if verbose:
            print(r.stdout + r.stderr)

    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        list(ex.map(run, jobs))
    if force or jobs or _stale(LIB, objs):
        run([nvcc(), *ARCH, "-shared", "-o", LIB, *objs])
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))

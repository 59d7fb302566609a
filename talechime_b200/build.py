"""Build libq8lin.so in-tree with nvcc for sm_100a.

    python -m talechime_b200.build        # or talechime_b200.build.build()

The library is written next to this file (talechime_b200/libq8lin.so) so that it
travels with the source tree; a JIT cache outside the tree is not used.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libq8lin.so")
OBJDIR = os.path.join(PKG, "_build")

SOURCES = ["abi.cu", "layout.cu", "gemv.cu", "gemm_simt.cu", "gemm_tc.cu", "noalloc.cu", "mlp.cu", "gemm_skinny.cu", "decoder.cu",
           "step.cu", "gemv_mrow.cu", "gguf.cpp", "tp_mlp.cu", "gemm_mma.cu", "prefill.cu"]
HEADERS = ["common.cuh", "internal.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    # IEEE division/reciprocal and no flush-to-zero: the Q8_0 scale arithmetic is
    # specified bit-exactly, so fast-math style flags must stay off.
    "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "q8lin.h")]
    objs = []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(OBJDIR, os.path.splitext(src)[0] + ".o")
        objs.append(obj)
        if force or _stale(obj, [path] + headers):
            cmd = [nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", path, "-o", obj]
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static",
               "-o", LIB, *objs, "-ldl"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv))

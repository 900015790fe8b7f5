"""Build libgpt2q.so in-tree with nvcc for sm_100a.

    python -m smelt_b200.build [--force] [--verbose-ptxas]

Objects go to smelt_b200/_build/, the library to smelt_b200/_lib/libgpt2q.so
(both git-ignored; the .so ships with the source tree to the GPU host).
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
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIBDIR, "libgpt2q.so")

SOURCES = ["kernels.cu", "runtime.cu", "gemm.cu", "gemm_mma.cu", "attn_tc.cu", "persistent.cu", "tp.cu", "noalloc.cu", "synth.cpp", "blake3.cpp", "smt.cpp", "backward.cu"]
HEADERS = ["common.cuh", "kernels.h", "gemm.h", "gemm_mma.h", "persistent.h", "tp.h", "tcgen05.cuh", "blake3.h", "backward.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _newer(src: list[str], dst: str) -> bool:
    if not os.path.exists(dst):
        return True
    t = os.path.getmtime(dst)
    return any(os.path.exists(s) and os.path.getmtime(s) > t for s in src)


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "gpt2q.h")]
    objs = []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s + ".o")
        objs.append(obj)
        if not (force or _newer([src, __file__] + hdrs, obj)):
            continue
        cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
               "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
        if verbose_ptxas and s.endswith(".cu"):
            cmd[1:1] = ["-Xptxas", "-v"]
        print("[smelt_b200.build]", " ".join(cmd[-3:]), flush=True)
        subprocess.run(cmd, check=True)
    if force or _newer(objs, LIB):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-ldl", "-lpthread"]
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose_ptxas="--verbose-ptxas" in sys.argv)
    print(LIB)

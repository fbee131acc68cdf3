"""Build the sm_100a backend library ``apeiron_b200/libapeiron_cuda.so`` in place.

nvcc cross-compiles for sm_100a without a GPU.  The library exports exactly the C ABI of
``include/apeiron_cuda.h``; cudart is linked statically so the file is self-contained.
Usage: ``python -m apeiron_b200.build`` (or ``build()`` from Python).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libapeiron_cuda.so")
SOURCES = ["apx_runtime.cu", "apx_gemv.cu", "apx_quant.cu", "apx_gemm.cu", "apx_lgemm.cu", "apx_ffn.cu",
           "apx_noalloc.cu",
           "apx_peer.cu", "apx_plan.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _objects_stale(srcs, lib) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(ROOT, "include", "apeiron_cuda.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra=None) -> str:
    srcs = [os.path.join(CSRC, s) for s in SOURCES if os.path.exists(os.path.join(CSRC, s))]
    if not force and not _objects_stale(srcs, LIB):
        return LIB
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-cudart=static",
           "-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp", *srcs]
    if extra:
        cmd[1:1] = list(extra)
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
    print(LIB)

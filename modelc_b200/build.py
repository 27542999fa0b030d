"""Build the sm_100a shared library ``libmodelc_cuda.so`` in-tree with nvcc.

The library is the product: hand-written CUDA kernels plus the C ABI declared
in ``include/modelc_cuda.h``.  It is compiled for sm_100a only.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libmodelc_cuda.so")
# Same sources with MC_TRACE: every launch of a captured verify records its
# first-CTA start, release from the dependency wait and last-CTA end
# (%globaltimer), plus per-phase times of the attention and tcgen05 kernels.
TRACE_LIB = os.path.join(HERE, "libmodelc_cuda_trace.so")
SOURCES = ["mc_kernels.cu", "mc_api.cu", "mc_drafters.cu", "mc_kvcache.cu"]
HEADERS = ["mc_internal.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(ROOT, "include", "modelc_cuda.h"))
    return any(os.path.getmtime(p) > t for p in deps)


def build(force: bool = False, verbose: bool = False, trace: bool = False) -> str:
    lib = TRACE_LIB if trace else LIB
    if not force and not _stale(lib):
        return lib
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           *(["-DMC_TRACE"] if trace else []),
           "-I", os.path.join(ROOT, "include"),
           *[os.path.join(CSRC, s) for s in SOURCES],
           "-o", lib + ".tmp", "-lcudart"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(lib + ".tmp", lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, trace="--trace" in sys.argv))

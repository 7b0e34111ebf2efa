"""Build libspruce_b200.so in-tree with nvcc for sm_100a.

    python -m spruce_research_b200.build          # or: python spruce_research_b200/build.py

The library is plain CUDA C++ with an extern "C" interface (include/spruce_b200.h);
it links the CUDA runtime statically and reaches the driver's tensor-map
encoder through cudaGetDriverEntryPoint, so it needs nothing but the driver
at run time.  Rebuilds only when a source is newer than the library.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libspruce_b200.so")
SOURCES = ["pool.cu", "select.cu", "tree.cu", "attn_sm100.cu", "attn_pair_sm100.cu", "attn_f32.cu",
           "summaries.cu", "residual.cu", "capi.cu"]
HEADERS = ["common.cuh", "kernels.h", "attn_common.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-shared", "-cudart", "static",
    "-Xptxas", "-v",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; install the CUDA toolkit to build libspruce_b200.so")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    built = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(REPO, "include", "spruce_b200.h"))
    return any(os.path.getmtime(d) > built for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if needed and return its path."""
    if not force and not _stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, "-I", os.path.join(REPO, "include"), "-o", tmp,
           *[os.path.join(CSRC, f) for f in SOURCES]]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("nvcc failed building libspruce_b200.so")
    if verbose:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))

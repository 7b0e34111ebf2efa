"""Build libspruce_b200.so in-tree with nvcc for sm_100a.

    python -m spruce_research_b200.build          # or: python spruce_research_b200/build.py

The library is plain CUDA C++ with an extern "C" interface (include/spruce_b200.h);
it links the CUDA runtime statically and reaches the driver's tensor-map
encoder through cudaGetDriverEntryPoint, so it needs nothing but the driver
at run time.  Rebuilds unless the library was built from exactly the current
sources, headers and flags (a SHA-256 kept beside it).
"""
from __future__ import annotations

import hashlib
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


KEY = LIB + ".key"  # SHA-256 of the sources, headers and flags the library was built from


def _source_key() -> str:
    h = hashlib.sha256()
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS] + [os.path.join(REPO, "include", "spruce_b200.h")]
    for d in deps:
        h.update(os.path.basename(d).encode())
        with open(d, "rb") as f:
            h.update(f.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def _stale() -> bool:
    """The library is rebuilt unless it exists and was built from exactly these sources and flags."""
    if not os.path.exists(LIB) or not os.path.exists(KEY):
        return True
    with open(KEY) as f:
        return f.read().strip() != _source_key()


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
    with open(KEY, "w") as f:
        f.write(_source_key() + "\n")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))

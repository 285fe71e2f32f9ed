"""Build the sm_100a shared library in-tree with nvcc.

    python -m ttjam_gottagofast_b200.build          # or build() from Python

The library (`libttjam_b200.so`, next to this file) holds every CUDA kernel of
the forward pass and the C ABI declared in include/ttjam_b200.h. It is built for
sm_100a only (`-gencode arch=compute_100a,code=sm_100a`); nvcc cross-compiles it
without a GPU.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_NAME = "libttjam_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)

SOURCES = ["api.cu", "layernorm.cu", "gemm_ffma.cu", "attention_ffma.cu", "cluster_forward.cu",
           "gemm_tc.cu", "attention_tc.cu", "noalloc.cu", "graph_cache.cu", "live_rows.cu",
           "tile_forward.cu", "typed_io.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build")
    return cand


def _sources():
    return [os.path.join(CSRC, s) for s in SOURCES]


def _headers():
    out = [os.path.join(ROOT, "include", "ttjam_b200.h")]
    out += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return out


def needs_rebuild() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(f) > t for f in _sources() + _headers())


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    if not force and not needs_rebuild():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, *(extra_flags or []),
           "-I", os.path.join(ROOT, "include"), "-I", CSRC,
           "-o", tmp, *_sources()]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra_flags=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
    print(LIB_PATH)

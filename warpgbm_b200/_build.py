"""Build libwgb_b200.so in-tree with nvcc for sm_100a.

    python -m warpgbm_b200._build          # or warpgbm_b200._build.build()

The library is plain C ABI (include/warpgbm_b200.h) linked against the
static CUDA runtime, so it loads next to any torch build.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libwgb_b200.so")
SOURCES = ["wgb_lib.cu", "wgb_engine.cu", "wgb_ops.cu", "wgb_io.cu", "wgb_quantile.cu", "wgb_noalloc.cu", "wgb_comm.cu", "wgb_decode.cu", "wgb_common.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-pthread", "-shared",
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    srcs.append(os.path.join(HERE, "..", "include", "warpgbm_b200.h"))
    return any(os.path.getmtime(s) > t for s in srcs if os.path.exists(s))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", tmp, os.path.join(CSRC, "wgb_lib.cu"), "-lpthread", "-ldl"]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))

"""Builds libvmscan.so (the sm_100a selective-scan library) in-tree.

Usage: ``python -m mlx_vision_mamba_b200.build`` or ``build()`` from Python.
The library is a single nvcc translation unit (csrc/vmscan.cu) with the CUDA
runtime linked statically, so it loads without a GPU and travels with the
source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_PATH = os.path.join(PKG_DIR, "libvmscan.so")
SOURCES = ["vmscan.cu"]
DEPS = ["vmscan.cu", "vmscan_common.cuh", "vmscan_fwd.cuh", "vmscan_bwd.cuh", "vmscan_conv.cuh", "vmscan_dt.cuh",
        "vmscan_gemm.cuh", "vmscan_norm.cuh"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libvmscan.so")
    return cand


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    root = os.path.dirname(PKG_DIR)
    deps = [os.path.join(CSRC, f) for f in DEPS] + [os.path.join(root, "include", "vmscan.h")]
    return any(os.path.getmtime(p) > t for p in deps if os.path.exists(p))


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    """Compile libvmscan.so for sm_100a if missing or out of date; return its path."""
    if not force and not _stale():
        return LIB_PATH
    cmd = [
        nvcc_path(),
        *ARCH_FLAGS,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-shared",
        "-Xcompiler",
        "-fPIC",
        "-cudart",
        "static",
        "-Xptxas",
        "-v" if verbose else "-O3",
        *(extra_flags or []),
        "-o",
        LIB_PATH + ".tmp",
        *[os.path.join(CSRC, s) for s in SOURCES],
    ]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + proc.stdout + proc.stderr)
    if verbose:
        sys.stdout.write(proc.stdout + proc.stderr)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))

"""Builds ``libconvrot.so`` (the sm_100a kernels and their C ABI) in-tree with nvcc.

``python -m hyperflow_h3_flash_b200.build`` or ``build()`` from Python. The library is written next to this file so
that it travels with a copy of the repository; nothing is installed elsewhere.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libconvrot.so")
SOURCES = sorted(os.path.join(HERE, "csrc", name) for name in os.listdir(os.path.join(HERE, "csrc"))
                 if name.endswith((".cu", ".cuh", ".h")))
HEADER = os.path.join(os.path.dirname(HERE), "include", "convrot.h")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    built = os.path.getmtime(LIB)
    return any(os.path.getmtime(src) > built for src in SOURCES + [HEADER])


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles the library if it is missing or older than its sources; returns its path."""
    if not force and not stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, "-o", tmp, os.path.join(HERE, "csrc", "convrot.cu")]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))

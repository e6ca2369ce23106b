"""In-tree build of the CUDA library (sm_100a) -- no JIT cache, the .so sits next to the
package so it travels with the source tree."""
from __future__ import annotations

import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libbitdance_b200.so")
SOURCES = [os.path.join(CSRC, "bitdance.cu")]
HEADERS = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-shared"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    inc = os.path.join(os.path.dirname(HERE), "include", "bitdance_b200.h")
    return any(os.path.getmtime(f) > t for f in SOURCES + HEADERS + [inc])


def build_library(force: bool = False, verbose: bool = False) -> str:
    if force or stale():
        cmd = [nvcc(), *NVCC_FLAGS, "-o", LIB, *SOURCES]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(r.stderr)
    return LIB

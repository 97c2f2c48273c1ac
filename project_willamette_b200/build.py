"""Build the sm_100a CUDA library in-tree.

    python -m project_willamette_b200.build [--ptxas-verbose]

Produces project_willamette_b200/_lib/libwillamette_b200.so: one nvcc
translation unit (csrc/willamette_b200.cu includes the kernel headers),
-gencode arch=compute_100a,code=sm_100a, cudart linked statically so the
library needs nothing beyond the driver at run time.  Cross-compiles on a
machine without a GPU.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "_lib")
LIB = os.path.join(LIBDIR, "libwillamette_b200.so")
MAIN = os.path.join(CSRC, "willamette_b200.cu")
HEADER = os.path.join(os.path.dirname(HERE), "include", "willamette_b200.h")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-cudart", "static",
    # IEEE division/sqrt and no FMA contraction across the explicit
    # __fmul_rn/__fadd_rn sequences the parity contract relies on.
    "-prec-div=true", "-prec-sqrt=true", "-fmad=false",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources() -> list[str]:
    out = [HEADER]
    for f in os.listdir(CSRC):
        if f.endswith((".cu", ".cuh", ".h")):
            out.append(os.path.join(CSRC, f))
    return out


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(s) <= t for s in _sources())


def build(force: bool = False, ptxas_verbose: bool = False) -> str:
    if not force and not ptxas_verbose and up_to_date():
        return LIB
    os.makedirs(LIBDIR, exist_ok=True)
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, "-o", tmp, MAIN]
    if ptxas_verbose:
        cmd[1:1] = ["-Xptxas", "-v"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force=True, ptxas_verbose="--ptxas-verbose" in sys.argv)
    print(LIB)

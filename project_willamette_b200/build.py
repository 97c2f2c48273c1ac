"""Build the sm_100a CUDA library in-tree.

    python -m project_willamette_b200.build [--ptxas-verbose]

Produces, from one nvcc translation unit (csrc/willamette_b200.cu includes
the kernel headers), -gencode arch=compute_100a,code=sm_100a:
  project_willamette_b200/_lib/libwillamette_b200.so -- cudart linked
      statically, so it needs nothing beyond the driver at run time (the
      Python package and the C client load it);
  project_willamette_b200/_lib/libwillamette_b200.a -- the same object as a
      static library, for a host program that links the C ABI into itself
      (a Rust build.rs: link it with cudart_static, rt, pthread, dl and
      stdc++).
Cross-compiles on a machine without a GPU.
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
STATIC_LIB = os.path.join(LIBDIR, "libwillamette_b200.a")
MAIN = os.path.join(CSRC, "willamette_b200.cu")
HEADER = os.path.join(os.path.dirname(HERE), "include", "willamette_b200.h")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
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
    if not os.path.exists(LIB) or not os.path.exists(STATIC_LIB):
        return False
    t = min(os.path.getmtime(LIB), os.path.getmtime(STATIC_LIB))
    return all(os.path.getmtime(s) <= t for s in _sources())


def build(force: bool = False, ptxas_verbose: bool = False) -> str:
    if not force and not ptxas_verbose and up_to_date():
        return LIB
    os.makedirs(LIBDIR, exist_ok=True)
    obj = os.path.join(LIBDIR, "willamette_b200.o")
    cmd = [nvcc(), *NVCC_FLAGS, "-c", "-o", obj, MAIN]
    if ptxas_verbose:
        cmd[1:1] = ["-Xptxas", "-v"]
    subprocess.run(cmd, check=True)
    tmp = LIB + ".tmp"
    subprocess.run([nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart",
                    "static", "-o", tmp, obj], check=True)
    os.replace(tmp, LIB)
    tmp_a = STATIC_LIB + ".tmp"
    if os.path.exists(tmp_a):
        os.remove(tmp_a)
    subprocess.run(["ar", "rcs", tmp_a, obj], check=True)
    os.replace(tmp_a, STATIC_LIB)
    os.remove(obj)
    return LIB


if __name__ == "__main__":
    build(force=True, ptxas_verbose="--ptxas-verbose" in sys.argv)
    print(LIB)

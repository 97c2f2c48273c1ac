"""The C ABI from a plain C client, no GPU needed: the header compiles as
strict C11 and as C++, and `c_consumer.c`, linked against the built library
the way a foreign-language binding links it, gets the reference's error
classes, empty-case results and zero-copy GGUF views through it."""
import os
import subprocess

import torch

from project_willamette_b200 import _abi

HERE = os.path.dirname(os.path.abspath(__file__))
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
STRICT = ["-Wall", "-Wextra", "-Werror", "-pedantic"]


def test_header_is_strict_c11_and_cxx(tmp_path):
    src = tmp_path / "h.c"
    src.write_text('#include "willamette_b200.h"\nint main(void) { return WL_OK; }\n')
    subprocess.run(["gcc", "-std=c11", *STRICT, "-I", INCLUDE, "-fsyntax-only", str(src)],
                   check=True, capture_output=True)
    subprocess.run(["g++", "-std=c++17", *STRICT, "-I", INCLUDE, "-fsyntax-only", "-x", "c++",
                    str(src)], check=True, capture_output=True)


def test_c_client_links_and_runs(tmp_path):
    _abi.lib()  # the library is built and loads
    libdir = os.path.dirname(_abi.LIB_PATH)
    exe = tmp_path / "c_consumer"
    r = subprocess.run(["gcc", "-std=c11", *STRICT, "-I", INCLUDE,
                        os.path.join(HERE, "c_consumer.c"), "-o", str(exe), "-L", libdir,
                        "-l:" + os.path.basename(_abi.LIB_PATH), "-Wl,-rpath," + libdir, "-lm"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    args = [] if torch.cuda.is_available() else ["--no-gpu"]
    r = subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr


def test_c_client_links_the_static_library(tmp_path):
    """The static library (what a Rust build.rs links into its binary) gives
    the same C client everything it needs: cudart linked statically, no
    shared library of ours at run time."""
    from project_willamette_b200 import build
    _abi.lib()
    assert os.path.exists(build.STATIC_LIB)
    cuda_lib = os.path.join(os.path.dirname(os.path.dirname(build.nvcc())), "lib64")
    exe = tmp_path / "c_consumer_static"
    r = subprocess.run(["gcc", "-std=c11", *STRICT, "-I", INCLUDE,
                        os.path.join(HERE, "c_consumer.c"), "-o", str(exe), build.STATIC_LIB,
                        "-L", cuda_lib, "-lcudart_static", "-lrt", "-lpthread", "-ldl", "-lstdc++",
                        "-lm"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run(["ldd", str(exe)], capture_output=True, text=True)
    assert "willamette" not in r.stdout and "cudart" not in r.stdout, r.stdout
    args = [] if torch.cuda.is_available() else ["--no-gpu"]
    r = subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr

"""The C ABI without Python: examples/c_forward.c (a C caller that allocates
with the CUDA runtime, sizes the buffers with mlora_*_bytes and calls
mlora_forward) compiles against include/mlora.h and libmlora.so on the CPU,
and on a GPU its forward matches its own plain-C restatement."""

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mini-tlora-reproduction_b200")
LIBDIR = os.path.join(PKG, "tlora_b200")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _compile(out_dir):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None or not os.path.exists(os.path.join(CUDA, "include", "cuda_runtime_api.h")):
        pytest.skip("no C compiler or CUDA headers")
    from tlora_b200 import _lib
    _lib.lib()  # builds / loads libmlora.so
    exe = os.path.join(out_dir, "c_forward")
    cmd = [cc, "-O2", os.path.join(PKG, "examples", "c_forward.c"), "-I" + os.path.join(ROOT, "include"),
           "-I" + os.path.join(CUDA, "include"), "-L" + LIBDIR, "-lmlora", "-Wl,-rpath," + LIBDIR,
           "-L" + os.path.join(CUDA, "lib64"), "-lcudart", "-Wl,-rpath," + os.path.join(CUDA, "lib64"), "-lm",
           "-o", exe]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return exe


def test_c_example_compiles_against_the_header(tmp_path):
    assert os.path.exists(_compile(str(tmp_path)))


@pytest.mark.gpu
def test_c_example_runs(tmp_path):
    exe = _compile(str(tmp_path))
    res = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "relative L2 error" in res.stdout

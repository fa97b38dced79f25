"""Build step of the native library: compiles csrc/ into tlora_b200/libmlora.so
for sm_100a with nvcc (works without a GPU; nvcc cross-compiles)."""

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
SRC_DIR = os.path.join(os.path.dirname(PKG_DIR), "csrc")
LIB_PATH = os.path.join(PKG_DIR, "libmlora.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr",
]


def _nvcc():
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the mlora CUDA library cannot be built")


def sources():
    return sorted(os.path.join(SRC_DIR, f) for f in os.listdir(SRC_DIR) if f.endswith((".cu", ".cuh")))


def up_to_date():
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    hdr = os.path.join(os.path.dirname(os.path.dirname(PKG_DIR)), "include", "mlora.h")
    return all(os.path.getmtime(s) <= t for s in sources() + [hdr, __file__])


def build(force=False, verbose=False, extra=()):
    if not force and up_to_date():
        return LIB_PATH
    cmd = [_nvcc(), *NVCC_FLAGS, *extra, "-o", LIB_PATH + ".tmp", os.path.join(SRC_DIR, "libmlora.cu")]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, file=sys.stderr)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=("-Xptxas", "-v") if "--ptxas" in sys.argv else ())
    print(LIB_PATH)

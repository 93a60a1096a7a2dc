"""Build the CUDA engine library `libchonk_b200.so` in-tree for sm_100a.

Plain nvcc, no torch extension: the library exports only the C ABI declared
in include/chonk_b200.h and links the CUDA runtime statically.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "libchonk_b200.so")
SOURCES = [os.path.join(PKG, "csrc", "ck_engine.cu")]
DEPS = sorted(glob.glob(os.path.join(PKG, "csrc", "*.cu*"))) + [os.path.join(ROOT, "include", "chonk_b200.h")]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
         "-shared", "-cudart", "static"]


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    tmp = LIB + f".tmp{os.getpid()}"
    cmd = [NVCC, *FLAGS, "-o", tmp, *SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)

# -*- coding: utf-8 -*-
"""Build libptq8.so (sm_100a) in-tree with nvcc.

    python -m ptq_int8_lab_b200.build

The library is plain CUDA runtime + C++ (no torch linkage); the Python host
side loads it with ctypes.  Output: ptq_int8_lab_b200/_lib/libptq8.so.
"""
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "csrc"
OUT = HERE / "_lib"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def _run(cmd):
    print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)


def build(verbose_ptxas: bool = False) -> Path:
    OUT.mkdir(exist_ok=True)
    lib = OUT / "libptq8.so"
    objs = []
    common = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(HERE.parent / "include")]
    o1 = OUT / "ptq8_model.o"
    _run([NVCC, *common, *ARCH, "-x", "c++", "-c", str(SRC / "ptq8_model.cpp"), "-o", str(o1)])
    objs.append(o1)
    o2 = OUT / "ptq8_engine.o"
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    _run([NVCC, *common, *ARCH, "-lineinfo", *extra, "-c", str(SRC / "ptq8_engine.cu"), "-o", str(o2)])
    objs.append(o2)
    tmp = OUT / "libptq8.so.tmp"
    _run([NVCC, "-shared", *ARCH, *[str(o) for o in objs], "-o", str(tmp), "-lcudart"])
    os.replace(tmp, lib)
    for o in objs:
        o.unlink()
    return lib


if __name__ == "__main__":
    build(verbose_ptxas="-v" in sys.argv)

"""Builds hanns_b200/lib/libhanns_gpu.so (sm_100a) with nvcc, in-tree.

    python -m hanns_b200.build [--force]

Every CUDA source is compiled with --fmad=false (the reference's Rust float code is
never contracted; fused multiply-adds are written explicitly where the reference
fuses) and IEEE division / square root.  cudart is linked statically so the library
loads with ctypes without any LD_LIBRARY_PATH.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(OUT_DIR, "libhanns_gpu.so")
OBJ_DIR = os.path.join(HERE, "_build")

CU_SOURCES = ["search_kernels.cu", "build_kernels.cu", "ivf_usq_gpu.cu", "capi.cu",
              "coarse_static.cu", "coarse_tc.cu", "scan_tc.cu"]
CPP_SOURCES = ["rotation.cpp", "ivfusq00.cpp"]
HEADERS = ["common.cuh", "kernels.h", "ivf_usq_gpu.h", "warp_select.cuh"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def cxx() -> str:
    return "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    inc = ["-I", CSRC, "-I", os.path.join(ROOT, "include")]
    common_deps = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "hanns_gpu.h")]
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ_DIR, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + common_deps):
            cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "--fmad=false",
                   "-prec-div=true", "-prec-sqrt=true", "-Xcompiler", "-fPIC",
                   "-ccbin", cxx(), *inc, "-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd))
            subprocess.run(cmd, check=True)
    for src in CPP_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ_DIR, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + common_deps):
            cmd = [cxx(), "-O2", "-std=c++17", "-fPIC", "-fopenmp", *inc, "-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd))
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-ccbin", cxx(), "-o", LIB, *objs,
               "-Xcompiler", "-fopenmp", "-lgomp"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    sys.exit(0)

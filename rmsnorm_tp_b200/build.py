"""Build the C-ABI shared library ``librmsnorm_tp_b200.so`` in-tree for sm_100a.

The library is plain CUDA C++ (no torch, no pybind11): kernels.cu holds the
forward kernels and their launcher, backward.cu the backward kernels,
noalloc.cu the allocation-free group entry point, linear.cu the fused row-parallel linear
(tcgen05 GEMM) -> reduce-scatter -> TP RMSNorm kernel, comm.cpp the extern "C" entry points declared in
include/rmsnorm_tp_b200.h. The CUDA runtime is linked statically, so the
library loads (and its symbols can be listed) on a machine without a GPU.

    python rmsnorm_tp_b200/build.py          # build if sources are newer
    python rmsnorm_tp_b200/build.py --force  # always rebuild

(Run it as a file: importing the package loads the library it builds.)
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
OUT_DIR = os.path.join(PKG_DIR, "_C")
LIB_NAME = "librmsnorm_tp_b200.so"
LIB_PATH = os.path.join(OUT_DIR, LIB_NAME)

SOURCES = [os.path.join(CSRC, "kernels.cu"), os.path.join(CSRC, "backward.cu"),
           os.path.join(CSRC, "comm.cpp"), os.path.join(CSRC, "noalloc.cu"),
           os.path.join(CSRC, "linear.cu")]
HEADERS = [
    os.path.join(CSRC, "device_common.cuh"),
    os.path.join(CSRC, "rtp_common.h"),
    os.path.join(CSRC, "internal.h"),
    os.path.join(CSRC, "ptx.cuh"),
    os.path.join(CSRC, "sm100.cuh"),
    os.path.join(ROOT_DIR, "include", "rmsnorm_tp_b200.h"),
]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-Wall",
    "-shared",
    "-cudart", "static",
]


def find_nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin directory on PATH")


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(p) > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if it is missing or older than its sources; return its path."""
    if not force and not needs_build():
        return LIB_PATH
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [find_nvcc(), *NVCC_FLAGS, "-I", os.path.join(ROOT_DIR, "include"), "-o", tmp, *SOURCES]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""Compile the reference's fused kernel and its pybind11 binding, as shipped,
into oracle/_ref/ -- test and measurement infrastructure only.

Sources (read where they lie, never copied): csrc/rmsnorm_tp.cu and
csrc/bindings.cpp of a haowen-han/RmsnormTP checkout. The result is the
reference's own extension module ``rmsnorm_tp_cpp`` (CommBuffer, IpcHandle,
launch_fused_rmsnorm), built for ``compute_100/sm_100`` exactly as the
reference's setup.py targets Blackwell (setup.py:20-21), with nvcc and g++
invoked directly (the reference's setup.py is not run). It is the "reference
fused kernel" comparator of the benchmark; it handles fp32 only.

    python oracle/build_ref.py --reference <checkout>

oracle/_ref/ is git-ignored; the built module travels to the GPU box with the
working tree.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("RMSNORM_TP_REFERENCE"),
                    help="checkout of the reference (default: $RMSNORM_TP_REFERENCE)")
    ap.add_argument("--nvcc", default="nvcc")
    args = ap.parse_args(argv)
    if not args.reference:
        print("no reference checkout given (--reference or RMSNORM_TP_REFERENCE); nothing to build")
        return 0
    csrc = os.path.join(args.reference, "csrc")
    if not os.path.isdir(csrc):
        print(f"no reference checkout at {args.reference}; nothing to build")
        return 0

    import torch
    from torch.utils import cpp_extension

    os.makedirs(OUT, exist_ok=True)
    inc = cpp_extension.include_paths(device_type="cuda") if "device_type" in \
        cpp_extension.include_paths.__code__.co_varnames else cpp_extension.include_paths(cuda=True)
    incs = [f"-I{p}" for p in inc] + [f"-I{sysconfig.get_paths()['include']}", f"-I{csrc}"]
    libdirs = cpp_extension.library_paths(device_type="cuda") if "device_type" in \
        cpp_extension.library_paths.__code__.co_varnames else cpp_extension.library_paths(cuda=True)
    abi = f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"
    defs = ["-DTORCH_EXTENSION_NAME=rmsnorm_tp_cpp", "-DTORCH_API_INCLUDE_EXTENSION_H", abi]
    ext = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    so = os.path.join(OUT, "rmsnorm_tp_cpp" + ext)
    cu_obj = os.path.join(OUT, "rmsnorm_tp.o")
    cpp_obj = os.path.join(OUT, "bindings.o")

    nvcc_cmd = [args.nvcc, "-c", os.path.join(csrc, "rmsnorm_tp.cu"), "-o", cu_obj,
                "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                "--generate-code=arch=compute_100,code=[compute_100,sm_100]", *defs, *incs]
    cxx_cmd = ["g++", "-c", os.path.join(csrc, "bindings.cpp"), "-o", cpp_obj, "-O3", "-std=c++17",
               "-fPIC", *defs, *incs]
    link_cmd = ["g++", "-shared", "-o", so, cpp_obj, cu_obj,
                *[f"-L{d}" for d in libdirs], *[f"-Wl,-rpath,{d}" for d in libdirs],
                "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
                "-lcudart"]
    for cmd in (nvcc_cmd, cxx_cmd, link_cmd):
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            print(" ".join(cmd))
            print(res.stdout[-4000:], res.stderr[-4000:])
            return res.returncode
    for p in (cu_obj, cpp_obj):
        os.unlink(p)
    print(so)
    return 0


if __name__ == "__main__":
    sys.exit(main())

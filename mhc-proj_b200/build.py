"""Build the native parts of mhc_proj in place.

    python mhc-proj_b200/build.py            # build what is out of date
    python mhc-proj_b200/build.py --force    # rebuild everything

Products, written next to the Python package so they travel with the tree:
  mhc_proj/libmhcproj.so        CUDA kernels + the C ABI of include/mhc_proj.h
                                (nvcc, sm_100a only)
  mhc_proj/_internal*.so        the PyTorch binding (pybind11), linked to
                                libmhcproj.so through an $ORIGIN rpath
Object files go to _build/.
"""
from __future__ import annotations

import argparse
import os
import shlex
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
PKG = os.path.join(HERE, "mhc_proj")
BUILD = os.path.join(HERE, "_build")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"

COMMON_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
]
# Per-source math flags.  The Newton kernels take --use_fast_math, as the
# reference's build does (setup.py:28), so their exp/log/divide give its
# results exactly.  The Sinkhorn-Knopp kernels use only explicitly rounded
# operations and a correctly rounded reciprocal; they keep the reference's
# flush-to-zero but take the accurate expf for the fused exp(R) kernels.
CU_SOURCES = {
    "birkhoff_n4.cu": ["--use_fast_math"],
    "sinkhorn_n4.cu": ["-ftz=true", "-prec-div=true", "-prec-sqrt=true", "-fmad=true"],
}

LIB = os.path.join(PKG, "libmhcproj.so")
EXT = os.path.join(PKG, "_internal" + sysconfig.get_config_var("EXT_SUFFIX"))


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print("+", " ".join(shlex.quote(c) for c in cmd), flush=True)
    subprocess.run(cmd, check=True)


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(INCLUDE, "mhc_proj.h")]


def build_cuda_lib(force: bool = False, verbose: bool = True) -> str:
    os.makedirs(BUILD, exist_ok=True)
    objs = []
    for src, math_flags in CU_SOURCES.items():
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        if force or _stale(o, [s, *_headers(), __file__]):
            _run([NVCC, *COMMON_FLAGS, *math_flags, "-I", INCLUDE, "-I", CSRC, "-c", s, "-o", o], verbose)
        objs.append(o)
    if force or _stale(LIB, objs):
        _run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", LIB,
              "-lcudart", "-Xlinker", "-soname=libmhcproj.so"], verbose)
    return LIB


def build_torch_ext(force: bool = False, verbose: bool = True) -> str:
    src = os.path.join(CSRC, "torch_binding.cpp")
    if not (force or _stale(EXT, [src, LIB, os.path.join(INCLUDE, "mhc_proj.h"), __file__])):
        return EXT
    import torch
    from torch.utils import cpp_extension as ce

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    flags = ["-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
             f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
             "-DTORCH_EXTENSION_NAME=_internal", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    incs = []
    for p in ce.include_paths(device_type="cuda"):
        incs += ["-isystem", p]
    incs += ["-isystem", sysconfig.get_paths()["include"], "-I", INCLUDE]
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    libs = ["-L", torch_lib, "-Wl,-rpath," + torch_lib,
            "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
            "-L", os.path.join(CUDA_HOME, "lib64"), "-lcudart",
            "-L", PKG, "-l:libmhcproj.so", "-Wl,-rpath,$ORIGIN"]
    _run([CXX, *flags, *incs, src, "-o", EXT, *libs], verbose)
    return EXT


def build(force: bool = False, verbose: bool = True) -> None:
    build_cuda_lib(force, verbose)
    build_torch_ext(force, verbose)


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-q", "--quiet", action="store_true")
    a = ap.parse_args()
    build(force=a.force, verbose=not a.quiet)
    sys.exit(0)

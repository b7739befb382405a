"""Build the native parts of the package in-tree.

* ``lib/libdcn_b200.so`` -- the CUDA library (all kernels + the C ABI of
  ``include/dcn_b200.h``), compiled by nvcc for sm_100a only;
* ``lib/libdcn_b200_torch.so`` -- the PyTorch operator registration
  (``csrc/torch_ops.cpp``), linked against the library above.

Run ``python -m pytorch_mps_deform_conv2d_b200._build`` (or
``__graft_entry__.build()``).  Objects are rebuilt only when a source or
header is newer than the library.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIBDIR = os.path.join(PKG, "lib")
OBJDIR = os.path.join(PKG, "_build", "obj")

LIB = os.path.join(LIBDIR, "libdcn_b200.so")
TORCH_LIB = os.path.join(LIBDIR, "libdcn_b200_torch.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
                     "-Xcompiler", "-fPIC,-fvisibility=hidden",
                     "-I" + INCLUDE, "-I" + CSRC]


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def _newest(paths) -> float:
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def _cu_sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
            glob.glob(os.path.join(INCLUDE, "*.h")))


def build_library(verbose: bool = False, force: bool = False) -> str:
    """Compile every ``csrc/*.cu`` for sm_100a and link ``lib/libdcn_b200.so``."""
    os.makedirs(OBJDIR, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    sources = _cu_sources()
    hdr_time = _newest(_headers())
    jobs = []
    for src in sources:
        obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr_time):
            jobs.append((src, obj))

    def compile_one(job):
        src, obj = job
        cmd = [_nvcc()] + NVCC_FLAGS + ["-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
        if verbose and (res.stdout or res.stderr):
            print(res.stdout + res.stderr, flush=True)
        return obj

    with cf.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        list(ex.map(compile_one, jobs))
    objs = [os.path.join(OBJDIR, os.path.basename(s) + ".o") for s in sources]
    if force or jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        cmd = [_nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def build_torch_ops(verbose: bool = False, force: bool = False) -> str:
    """Compile ``csrc/torch_ops.cpp`` against PyTorch into ``lib/libdcn_b200_torch.so``."""
    src = os.path.join(CSRC, "torch_ops.cpp")
    if (not force and os.path.exists(TORCH_LIB) and
            os.path.getmtime(TORCH_LIB) >= max(os.path.getmtime(src), os.path.getmtime(LIB),
                                              _newest(_headers()))):
        return TORCH_LIB
    import torch
    from torch.utils import cpp_extension

    os.makedirs(LIBDIR, exist_ok=True)
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = cpp_extension.include_paths(device_type="cuda") + [os.path.join(cuda, "include"),
                                                               INCLUDE, CSRC]
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    cmd = (["g++", "-shared", "-fPIC", "-O2", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
            "-DTORCH_API_INCLUDE_EXTENSION_H"] + ["-I" + i for i in incs] +
           [src, "-o", TORCH_LIB, "-L" + torch_lib, "-lc10", "-lc10_cuda", "-ltorch_cpu",
            "-ltorch_cuda", "-ltorch", "-L" + os.path.join(cuda, "lib64"), "-lcudart",
            "-L" + LIBDIR, "-ldcn_b200", "-Wl,-rpath,$ORIGIN"])
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed on {src}:\n{res.stdout}\n{res.stderr}")
    return TORCH_LIB


def build_all(verbose: bool = False, force: bool = False) -> None:
    build_library(verbose=verbose, force=force)
    build_torch_ops(verbose=verbose, force=force)


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv, force="--force" in sys.argv)
    print(LIB)
    print(TORCH_LIB)

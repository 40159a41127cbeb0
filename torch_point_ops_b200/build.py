"""In-tree build of the tpo_b200 native libraries (sm_100a).

Produces, inside the package directory:
  lib/libtpo_b200.so       CUDA kernels + the extern "C" boundary (include/tpo_b200.h);
                           depends only on the CUDA driver (cudart linked statically).
  lib/libtpo_b200_torch.so torch.library binding over that C ABI.

Usage:  python torch_point_ops_b200/build.py [--force]   (run as a script: importing
        the package itself requires the built libraries)
Incremental: a target is rebuilt when any of its sources or headers is newer.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "lib")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

CU_SOURCES = ["chamfer_fwd.cu", "chamfer_bwd.cu", "knn.cu", "capi.cu", "chamfer_noalloc.cu", "gather_points.cu", "fps.cu",
              "pipe_probe.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
]
CAPI_LIB = os.path.join(LIB, "libtpo_b200.so")
TORCH_LIB = os.path.join(LIB, "libtpo_b200_torch.so")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(
        os.path.join(ROOT, "include", "*.h"))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout)
    return r.stdout


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIB, exist_ok=True)
    hdrs = _headers()
    jobs = []
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            jobs.append([NVCC] + NVCC_FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-c", s, "-o", o])
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        for out in ex.map(_run, jobs):
            if verbose and out:
                print(out)
    if force or _stale(CAPI_LIB, objs):
        # cudart static: the library needs nothing but the driver; it interoperates
        # with torch through plain device pointers and cudaStream_t handles.
        _run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static",
              "-o", CAPI_LIB] + objs)

    # torch binding (host-only C++), linked against the C ABI library.
    import torch
    from torch.utils import cpp_extension as ce

    src = os.path.join(CSRC, "torch_ops.cpp")
    if force or _stale(TORCH_LIB, [src, CAPI_LIB] + hdrs):
        tdir = os.path.dirname(torch.__file__)
        inc = [f"-I{p}" for p in ce.include_paths()] + [f"-I{os.path.join(CUDA_HOME, 'include')}",
                                                        f"-I{sysconfig.get_paths()['include']}"]
        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
              src, "-o", TORCH_LIB] + inc + [
              f"-L{LIB}", "-ltpo_b200", f"-L{os.path.join(tdir, 'lib')}",
              "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch",
              "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{os.path.join(tdir, 'lib')}"])
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print("built", CAPI_LIB, TORCH_LIB)

"""In-tree build of the two native libraries of rapidadb_b200.

* ``librdb_kernels.so`` - every ``csrc/*.cu`` compiled by nvcc for sm_100a
  (``-gencode arch=compute_100a,code=sm_100a``), static CUDA runtime; it
  exports the C ABI of ``include/rapidadb_b200.h`` and nothing needs torch.
* ``_C.so`` - the C++ host layer (``csrc/host/*.cpp``, index classes +
  pybind11 bindings) linked against libtorch and ``librdb_kernels.so``
  (found next to it through ``$ORIGIN``).

Both land inside the package directory, so a copy of the source tree carries
them.  Rebuilds are incremental (object newer than its source and every
header).  ``python -m rapidadb_b200.build`` builds both.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
KERNEL_LIB = os.path.join(PKG, "librdb_kernels.so")
EXT_LIB = os.path.join(PKG, "_C.so")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC]
CXX = "g++"


def _headers():
    return (glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True)
            + glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True)
            + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed ({r.returncode}):\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r


def _torch_flags():
    import torch
    from torch.utils import cpp_extension as ce

    inc = ["-I" + p for p in ce.include_paths("cuda")]
    inc.append("-I" + sysconfig.get_paths()["include"])
    libdir = ce.library_paths("cuda")[0]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = ["-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
    libs = ["-L" + libdir, "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
            "-ltorch_python", "-Wl,-rpath," + libdir]
    return inc, defs, libs


def build_kernels(verbose=False, jobs=8):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = _headers()
    objs, todo = [], []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        if _stale(o, [s] + hdrs):
            todo.append([NVCC] + NVCC_FLAGS + ["-c", s, "-o", o])
    with ThreadPoolExecutor(jobs) as ex:
        list(ex.map(lambda c: _run(c, verbose), todo))
    if todo or _stale(KERNEL_LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-cudart", "static", "-Xcompiler", "-fPIC"] + objs
             + ["-o", KERNEL_LIB], verbose)
    return KERNEL_LIB


def build_extension(verbose=False, jobs=8):
    os.makedirs(BUILD, exist_ok=True)
    inc, defs, libs = _torch_flags()
    srcs = sorted(glob.glob(os.path.join(CSRC, "host", "*.cpp")))
    hdrs = _headers()
    objs, todo = [], []
    for s in srcs:
        o = os.path.join(BUILD, "host_" + os.path.basename(s) + ".o")
        objs.append(o)
        if _stale(o, [s] + hdrs):
            todo.append([CXX, "-O2", "-std=c++17", "-fPIC", "-I" + INCLUDE, "-I" + CSRC]
                        + inc + defs + ["-c", s, "-o", o])
    with ThreadPoolExecutor(jobs) as ex:
        list(ex.map(lambda c: _run(c, verbose), todo))
    if todo or _stale(EXT_LIB, objs + [KERNEL_LIB]):
        _run([CXX, "-shared", "-o", EXT_LIB] + objs
             + ["-L" + PKG, "-lrdb_kernels", "-Wl,-rpath,$ORIGIN"] + libs, verbose)
    return EXT_LIB


def build(verbose=False):
    build_kernels(verbose)
    build_extension(verbose)
    return KERNEL_LIB, EXT_LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print("built", KERNEL_LIB, EXT_LIB)

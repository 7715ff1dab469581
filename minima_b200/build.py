"""Build the in-tree native libraries of minima_b200.

* libminima_cuda.so      CUDA token loop + C ABI (include/minima_cuda.h),
                         nvcc for sm_100a only.
* libminima_generate.so  drop-in generate.h implementation (C) over it.
* libminima_forward.so   drop-in forward.h implementation (C) over it.
* libminima_host.so      model init / arena / RNG for standalone programs.

Outputs stay next to the sources (not installed), so that the files a GPU
run loads are the ones built here.  Rebuilds only what is out of date.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
INC = os.path.join(ROOT, "include")
CSRC = os.path.join(PKG, "csrc")
HOST = os.path.join(PKG, "host")

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
# The image's CC variable points at a gcc wrapper without OpenMP; use the system gcc.
GCC = "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

LIB_CUDA = os.path.join(PKG, "libminima_cuda.so")
LIB_GEN = os.path.join(PKG, "libminima_generate.so")
LIB_HOST = os.path.join(PKG, "libminima_host.so")
LIB_FWD = os.path.join(PKG, "libminima_forward.so")


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def _files(d, exts):
    return [os.path.join(d, f) for f in sorted(os.listdir(d)) if f.endswith(exts)]


def build(verbose: bool = False, force: bool = False) -> None:
    cuda_deps = _files(CSRC, (".cu", ".cuh")) + _files(INC, (".h",))
    if force or _stale(LIB_CUDA, cuda_deps):
        _run([NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-O2", "-shared", f"-I{INC}", "-o", LIB_CUDA,
              os.path.join(CSRC, "minima_cuda.cu"), "-lcudart"], verbose)
    gen_src = os.path.join(HOST, "generate_cuda.c")
    if force or _stale(LIB_GEN, [gen_src, LIB_CUDA] + _files(INC, (".h",))):
        _run([GCC, "-std=c11", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra", f"-I{INC}",
              "-o", LIB_GEN, gen_src, f"-L{PKG}", "-lminima_cuda", "-Wl,-rpath,$ORIGIN",
              "-lm"], verbose)
    fwd_src = os.path.join(HOST, "forward_cuda.c")
    if force or _stale(LIB_FWD, [fwd_src, LIB_GEN, LIB_CUDA] + _files(INC, (".h",))):
        _run([GCC, "-std=c11", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra", f"-I{INC}",
              "-o", LIB_FWD, fwd_src, f"-L{PKG}", "-lminima_generate", "-lminima_cuda",
              "-Wl,-rpath,$ORIGIN", "-lm"], verbose)
    host_src = os.path.join(HOST, "host_support.c")
    if force or _stale(LIB_HOST, [host_src] + _files(INC, (".h",))):
        _run([GCC, "-std=c11", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra", f"-I{INC}",
              "-o", LIB_HOST, host_src, "-lm"], verbose)


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)

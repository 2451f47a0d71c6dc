"""Builds the native libraries of the package in-tree.

* ``libkx.so``            — the sm_100a kernels behind the kx C ABI (include/kx.h),
                            compiled with nvcc for ``arch=compute_100a,code=sm_100a``.
* ``libgpu_scheduler.so`` — the LD_PRELOAD interposer + HP/BE scheduler
                            (C++; exports the reference's cuBLAS / cuDNN / CUDA
                            runtime / orion_* symbols).

Objects are compiled in parallel and cached by source mtime under
``kernel_intercept_b200/_build``.  ``python -m kernel_intercept_b200.build``
builds everything.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
SHIM = os.path.join(CSRC, "shim")
INC = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")
CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "--expt-relaxed-constexpr", "-ccbin", CXX, "-I" + INC, "-I" + CSRC]

LIBKX = os.path.join(PKG, "libkx.so")
LIBSHIM = os.path.join(PKG, "libgpu_scheduler.so")


def _deps(src: str) -> list[str]:
    hdrs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INC, "*.h"))
    if os.path.dirname(src) == SHIM:
        hdrs += glob.glob(os.path.join(SHIM, "*.h"))
    return [src] + hdrs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {os.path.basename(cmd[-1])}")


def _compile_cu(src: str, extra: list[str] | None = None) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if _stale(obj, _deps(src)):
        _run([NVCC] + NVCC_FLAGS + (extra or []) + ["-c", "-o", obj, src])
    return obj


def build_kx(jobs: int | None = None, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    extra = ["-Xptxas", "-v"] if verbose_ptxas else None
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile_cu(s, extra), srcs))
    if _stale(LIBKX, objs + [os.path.join(CSRC, "kx.map")]):
        tmp = LIBKX + ".tmp"
        _run([NVCC] + ARCH + ["-shared", "-cudart", "static", "-ccbin", CXX, "-o", tmp] + objs +
             ["-Xlinker", "--version-script=" + os.path.join(CSRC, "kx.map"), "-ldl",
              "-lpthread"])
        os.replace(tmp, LIBKX)
    return LIBKX


def build_shim() -> str | None:
    srcs = sorted(glob.glob(os.path.join(SHIM, "*.cpp")))
    if not srcs:
        return None
    os.makedirs(BUILD, exist_ok=True)
    objs = []
    flags = ["-std=c++17", "-O2", "-fPIC", "-Wall", "-Wno-unused-parameter", "-I" + INC,
             "-I" + SHIM, "-I" + os.path.join(CUDA, "include")]
    for s in srcs:
        obj = os.path.join(BUILD, "shim_" + os.path.basename(s) + ".o")
        if _stale(obj, _deps(s)):
            _run([CXX] + flags + ["-c", "-o", obj, s])
        objs.append(obj)
    if _stale(LIBSHIM, objs + [LIBKX]):
        tmp = LIBSHIM + ".tmp"
        # No link against cudart / cuBLAS / cuDNN: the real functions are
        # looked up at run time (dlsym), kx through its C ABI.
        _run([CXX, "-shared", "-o", tmp] + objs +
             ["-L" + PKG, "-lkx", "-Wl,-rpath,$ORIGIN", "-ldl", "-lpthread"])
        os.replace(tmp, LIBSHIM)
    return LIBSHIM


def build_all() -> None:
    build_kx()
    build_shim()


def clean() -> None:
    shutil.rmtree(BUILD, ignore_errors=True)
    for f in (LIBKX, LIBSHIM):
        if os.path.exists(f):
            os.remove(f)


if __name__ == "__main__":
    if "--clean" in sys.argv:
        clean()
    build_kx(verbose_ptxas="--ptxas-v" in sys.argv)
    build_shim()
    print(LIBKX)

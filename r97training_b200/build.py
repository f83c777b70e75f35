"""Builds libr97b200.so (the sm_100a kernels and their C ABI) and libr97host.so (the C++ host side that
keeps the reference's adjoint-registry API) in-tree, with nvcc / g++. Run as
``python -m r97training_b200.build``; ``__graft_entry__.build()`` calls :func:`build_all`.
"""
from __future__ import annotations

import concurrent.futures
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
HOST = os.path.join(PKG, "host")
OBJ = os.path.join(ROOT, "_build", "obj")
LIB = os.path.join(PKG, "libr97b200.so")
HOSTLIB = os.path.join(PKG, "libr97host.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O3",
                  "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def _compile(src: str, headers) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if _newer(obj, [src] + headers):
        return obj
    cmd = [NVCC] + NVFLAGS + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build_kernels(verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) +
                     glob.glob(os.path.join(ROOT, "include", "*.h")))
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, headers), srcs))
    if not _newer(LIB, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-Xlinker", "-soname=libr97b200.so", "-o", LIB] + objs + ["-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        if verbose:
            print("built", LIB)
    return LIB


def build_host(verbose: bool = False) -> str:
    srcs = sorted(glob.glob(os.path.join(HOST, "*.cpp")))
    if not srcs:
        return ""
    headers = sorted(glob.glob(os.path.join(HOST, "*.h")) + glob.glob(os.path.join(ROOT, "include", "*.h")))
    if _newer(HOSTLIB, srcs + headers + [LIB]):
        return HOSTLIB
    # links the kernel library by name, found beside it at run time ($ORIGIN); the reference's registry
    # symbols stay weak and unresolved until a process that holds them loads the plugin
    cmd = ["g++", "-O2", "-std=c++20", "-fPIC", "-shared", "-pthread", "-I", os.path.join(ROOT, "include"),
           "-Wl,-soname,libr97host.so", "-o", HOSTLIB] + srcs + ["-L", PKG, "-lr97b200", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print("built", HOSTLIB)
    return HOSTLIB


def build_all(verbose: bool = False) -> None:
    build_kernels(verbose)
    build_host(verbose)


if __name__ == "__main__":
    build_all(verbose=True)
    sys.exit(0)

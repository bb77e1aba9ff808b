"""Build libfusiongpu_b200.so in-tree with nvcc for sm_100a, and the C++
programs on top of its C ABI.

    python -m fusiongpu_b200.build [--verbose] [--ptxas-v]

Each ``csrc/*.cu`` is compiled to an object in ``_build/`` (in parallel), then
linked into ``fusiongpu_b200/libfusiongpu_b200.so``.  Each ``host/*.cpp`` is
a program (fg_build_global, fg_search_pipeline, fg_tune_parameters) linked
against the library into ``fusiongpu_b200/bin/``.  Targets are rebuilt when
their source or any header changed.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libfusiongpu_b200.so")
HOST = os.path.join(PKG, "host")
BIN = os.path.join(PKG, "bin")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
HOST_CXX = os.environ.get("FG_HOST_CXX", "/usr/bin/g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-ccbin", HOST_CXX,
         "-I", os.path.join(ROOT, "include"), "-I", CSRC, "--expt-relaxed-constexpr"]


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, ptxas_v: bool, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if _stale(obj, [src, __file__] + _headers()):
        cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
        if ptxas_v:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if ptxas_v or verbose:
            sys.stdout.write(r.stderr)
    return obj


def _program(src: str, verbose: bool) -> str:
    exe = os.path.join(BIN, os.path.splitext(os.path.basename(src))[0])
    deps = [src, LIB, __file__] + glob.glob(os.path.join(HOST, "*.hpp")) + glob.glob(os.path.join(ROOT, "include", "*"))
    if _stale(exe, deps):
        cmd = [HOST_CXX, "-O2", "-std=c++17", "-Wall", "-pthread", "-I", os.path.join(ROOT, "include"), "-I", HOST,
               "-I", os.path.join(CUDA_HOME, "include"), src, "-o", exe, "-L", PKG, "-lfusiongpu_b200",
               "-L", os.path.join(CUDA_HOME, "lib64"), "-lcudart", "-Wl,-rpath,$ORIGIN/..",
               "-Wl,-rpath," + os.path.join(CUDA_HOME, "lib64")]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"g++ failed for {src}:\n{r.stdout}\n{r.stderr}")
    return exe


def programs(verbose: bool = False) -> list[str]:
    """Build the C++ programs (the library must be built)."""
    os.makedirs(BIN, exist_ok=True)
    return [_program(s, verbose) for s in sorted(glob.glob(os.path.join(HOST, "*.cpp")))]


def build(verbose: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, ptxas_v, verbose), srcs))
    if _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-ccbin", HOST_CXX, "-o", LIB, *objs, "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    programs(verbose)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose, a.ptxas_v))

"""Build libmrtdf.so (the engine's C ABI) in-tree for sm_100a.

    python magenta-realtime-mlx-cpp_b200/build.py [--force] [--verbose]

CUDA sources are compiled by nvcc with -gencode arch=compute_100a,code=sm_100a;
host C++ sources by g++; the shared library lands in
magenta-realtime-mlx-cpp_b200/lib/libmrtdf.so. The C++ dry-run driver
(cli/mrtdf_dry_run.cpp, built against include/mrtdf.hpp) lands beside it as
lib/mrtdf_dry_run. Objects are cached in _build/ and rebuilt when a source or
header is newer. No GPU is needed to build.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libmrtdf.so")
DRIVER_SRC = os.path.join(HERE, "cli", "mrtdf_dry_run.cpp")
DRIVER = os.path.join(LIBDIR, "mrtdf_dry_run")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(
        os.path.join(INCLUDE, "*.h")
    ) + glob.glob(os.path.join(INCLUDE, "*.hpp"))


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in _headers()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep:
        return obj
    if src.endswith(".cu"):
        cmd = [_nvcc(), "-std=c++17", "-O3", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC", "-Xptxas", "-v",
               "--expt-relaxed-constexpr", "-I", CSRC, "-c", src, "-o", obj]
    else:
        cmd = ["g++", "-std=c++17", "-O3", "-fPIC", "-Wall", "-I", CSRC, "-I", "/usr/local/cuda/include", "-c", src,
               "-o", obj]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    log = os.path.join(BUILD, os.path.basename(src) + ".log")
    with open(log, "w") as f:
        f.write(res.stdout + res.stderr)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"compile failed: {src}")
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    if force:
        for o in glob.glob(os.path.join(BUILD, "*.o")):
            os.remove(o)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), sources))
    if not (os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs)):
        tmp = LIB + ".tmp"
        cmd = [_nvcc(), "-shared", *ARCH, "-o", tmp, *objs, "-lcudart_static", "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.check_call(cmd)
        os.replace(tmp, LIB)
    build_driver(verbose)
    return LIB


def build_driver(verbose: bool = False) -> str:
    """The C++ dry-run driver, linked against libmrtdf.so (found next to it)."""
    newest = max([os.path.getmtime(DRIVER_SRC), os.path.getmtime(LIB)] + [os.path.getmtime(h) for h in _headers()])
    if os.path.exists(DRIVER) and os.path.getmtime(DRIVER) >= newest:
        return DRIVER
    tmp = DRIVER + ".tmp"
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-I", INCLUDE, DRIVER_SRC, "-o", tmp, "-L", LIBDIR, "-lmrtdf",
           "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("compile failed: " + DRIVER_SRC)
    os.replace(tmp, DRIVER)
    return DRIVER


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))

"""Build recipe for the CPU oracle (test infrastructure only).

Compiles the Depthformer, SpectroStream and MusicCoCa oracles (oracle/*.cpp) into
oracle/_build/liboracle.so with g++. The
exact-arithmetic translation unit (bf16 rounding, Philox, Gumbel, CFG mix)
is built with -ffp-contract=off so no multiply-add is fused; the model code
may fuse. -march=x86-64-v3 keeps the binary runnable on any AVX2 host, so it
can be built here and run on the GPU box.

The reference itself (rhymeswithlion/magenta-realtime-mlx-cpp) cannot be
compiled in this container: its CMakeLists.txt:23-28 requires MLX, which is
not installed, so there is no oracle/_ref build.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(BUILD, "liboracle.so")
SOURCES = ["depthformer_oracle.cpp", "oracle_exact.cpp", "spectrostream_oracle.cpp", "musiccoca_oracle.cpp"]
HEADERS = ["oracle.h", "safetensors_reader.h"]


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(os.path.join(HERE, f)) > t for f in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    common = ["g++", "-std=c++17", "-O3", "-march=x86-64-v3", "-fPIC", "-fopenmp", "-Wall", "-Wno-unused-function"]
    objs = []
    for src in SOURCES:
        obj = os.path.join(BUILD, src.replace(".cpp", ".o"))
        flags = list(common)
        if src == "oracle_exact.cpp":
            flags += ["-ffp-contract=off", "-fno-fast-math"]
        cmd = flags + ["-c", os.path.join(HERE, src), "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.check_call(cmd)
        objs.append(obj)
    tmp = LIB + ".tmp"
    subprocess.check_call(common + ["-shared", "-o", tmp] + objs)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))

"""Shared fixtures. `-m gpu` tests need a B200; everything else runs on CPU."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "magenta-realtime-mlx-cpp_b200")
ORACLE = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG, ORACLE, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def mrtdf():
    import build as pkg_build  # magenta-realtime-mlx-cpp_b200/build.py

    pkg_build.build()
    import mrtdf as m

    return m


@pytest.fixture(scope="session")
def oracle():
    import oracle_py

    oracle_py.lib()
    return oracle_py


@pytest.fixture(scope="session")
def tiny_weights(mrtdf, tmp_path_factory):
    """Random-init tiny bundle (seed 0, N(0, 0.02), norm scales 1)."""
    cfg = mrtdf.preset("tiny", mrtdf.DTYPE_FP32)
    path = str(tmp_path_factory.mktemp("w") / "depthformer_tiny.safetensors")
    mrtdf.write_random_safetensors(cfg, 0, path)
    return path


@pytest.fixture(scope="session")
def hybrid_weights(mrtdf, tmp_path_factory):
    """Random-init benchmark-architecture bundle (2.3 GB float32)."""
    cfg = mrtdf.preset("hybrid", mrtdf.DTYPE_FP32)
    path = str(tmp_path_factory.mktemp("wh") / "depthformer_hybrid.safetensors")
    mrtdf.write_random_safetensors(cfg, 0, path)
    return path


def random_ids(cfg, rows: int, seq_len: int, seed: int) -> np.ndarray:
    """Uniform ids; with rows == 2 the second (unconditioned) row has its
    last 6 (style) positions set to MASK = 1, as in system.cpp:91-93."""
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, cfg.vocab_size, size=(1, seq_len), dtype=np.int32)
    ids = np.repeat(ids, rows, axis=0)
    if rows == 2:
        ids[1, -6:] = 1
    return np.ascontiguousarray(ids)

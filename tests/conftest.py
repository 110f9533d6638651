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


# MusicCoCa text tower widths (musiccoca.h:151-162) and a reduced vocabulary
# for the random-init style bundles (the gather is the only place the
# vocabulary size enters).
STYLE_D, STYLE_H, STYLE_DH, STYLE_FF, STYLE_LAYERS, STYLE_POOL_DH = 768, 12, 64, 3072, 12, 256
STYLE_VOCAB, STYLE_LEVELS = 1000, 12


@pytest.fixture(scope="session")
def style_bundle(tmp_path_factory):
    """Random-init MusicCoCa text tower with the reference's key layout
    (musiccoca.cpp constructors) and a 12-level style codebook bundle, seed 90:
    (encoder path, codebooks path, {key: array})."""
    from safetensors.numpy import save_file

    D, H, DH, FF, POOL_DH = STYLE_D, STYLE_H, STYLE_DH, STYLE_FF, STYLE_POOL_DH
    rng = np.random.default_rng(90)
    w = {}

    def lin(p, out, inp):
        w[p + ".weight"] = (rng.standard_normal((out, inp)) / np.sqrt(inp)).astype(np.float32)
        w[p + ".bias"] = (rng.standard_normal(out) * 0.02).astype(np.float32)

    def ln(p):
        w[p + ".weight"] = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
        w[p + ".bias"] = (0.1 * rng.standard_normal(D)).astype(np.float32)

    w["token_embedding.weight"] = (rng.standard_normal((STYLE_VOCAB, D)) / np.sqrt(D)).astype(np.float32)
    for i in range(STYLE_LAYERS):
        p = f"text_layers.{i}"
        ln(p + ".attn_ln")
        ln(p + ".ffn_ln")
        for n in ("q", "k", "v"):
            lin(f"{p}.attn.{n}_proj", H * DH, D)
        lin(p + ".attn.o_proj", D, H * DH)
        lin(p + ".ffn_w1", FF, D)
        lin(p + ".ffn_w2", D, FF)
    ln("text_exit_ln")
    ln("text_pooler.ln")
    w["text_pooler.query"] = rng.standard_normal((1, 1, D)).astype(np.float32)
    for n in ("q", "k", "v"):
        lin(f"text_pooler.attn.{n}_proj", H * POOL_DH, D)
    lin("text_pooler.attn.o_proj", D, H * POOL_DH)
    w["text_pooler.attn._per_dim_scale"] = (0.5 * rng.standard_normal(POOL_DH)).astype(np.float32)
    d = tmp_path_factory.mktemp("style")
    enc, cb = str(d / "musiccoca_encoder.safetensors"), str(d / "musiccoca_codebooks.safetensors")
    save_file(w, enc)
    save_file({"codebooks": (rng.standard_normal((STYLE_LEVELS, 1024, D)) / np.sqrt(D)).astype(np.float32)}, cb)
    return enc, cb, w


def style_prompt(rng, n: int, vocab: int = STYLE_VOCAB):
    """StyleModel::tokenize_text_ids (style_model.cpp) layout: BOS = 1, then
    n pieces, zeros after; padding 1.0 on every position after them."""
    ids = np.zeros((1, 128), np.int32)
    pad = np.ones((1, 128), np.float32)
    ids[0, 0] = 1
    ids[0, 1:n + 1] = rng.integers(2, vocab, n)
    pad[0, :n + 1] = 0
    return ids, pad

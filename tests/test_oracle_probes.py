"""CPU checks of the oracle's own entry points used by the CPU arms and the
per-layer parity tests (no GPU, no compute in libmrtdf.so):

* the oracle's restated random-init generator builds the same weights as the
  engine's bundle writer (so the `--impl reference` arm never loads the
  engine library);
* its restated presets and encoder-input build equal the engine's;
* the single-layer probes compose to the whole-step entry points;
* frame-by-frame generation with the level-slice lm_head gives the tokens of
  the full-vocabulary path.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import random_ids


def test_presets_restated(mrtdf, oracle):
    for name in ("base", "large", "hybrid"):
        for dtype in (0, 1):
            assert oracle.preset_ints(name, dtype) == mrtdf.preset(name, dtype).as_ints(), name


def test_encoder_inputs_restated(mrtdf, oracle):
    rng = np.random.default_rng(3)
    for trial in range(20):
        F, D = int(rng.integers(1, 300)), 16
        ctx = rng.integers(-1, 1024, size=(F, D)).astype(np.int32)
        style = rng.integers(2, 16386, size=int(rng.integers(0, 8))).astype(np.int32)
        enc_depth = int(rng.integers(1, D + 1))
        np.testing.assert_array_equal(oracle.build_encoder_inputs(ctx, style, enc_depth, 1024, 2),
                                      mrtdf.build_encoder_inputs(ctx, style, enc_depth, 1024, 2))


@pytest.mark.parametrize("dtype", [0, 1])
def test_random_generator_restated(mrtdf, oracle, tiny_weights, dtype):
    """Oracle.from_random (in memory) == the bundle the engine's writer made."""
    cfg = mrtdf.preset("tiny", dtype)
    a = oracle.Oracle(tiny_weights, cfg.as_ints())
    b = oracle.Oracle.from_random(cfg.as_ints(), 0)
    ids = random_ids(cfg, 2, cfg.max_encoder_length, seed=5)
    toks = (cfg.codec_offset + np.arange(cfg.rvq_depth) * cfg.codebook_size + 7)[None].astype(np.int32)
    np.testing.assert_array_equal(a.teacher_forced(ids, toks, 1), b.teacher_forced(ids, toks, 1))


@pytest.mark.parametrize("dtype", [0, 1])
def test_layer_probes_compose(mrtdf, oracle, tiny_weights, dtype):
    """The decoder-layer probes chained over a stack reproduce temporal_step
    and depth_step bit for bit (same caches, same inputs), lm_head rows equal
    depth_step's logits, and the encoder-layer chain from embed_pe stays
    finite (it feeds encode, checked against the engine elsewhere)."""
    cfg = mrtdf.preset("tiny", dtype)
    ids = random_ids(cfg, 2, 40, seed=6)
    whole = oracle.Oracle(tiny_weights, cfg.as_ints())
    parts = oracle.Oracle(tiny_weights, cfg.as_ints())
    whole.encode(ids)
    parts.encode(ids)
    x = parts.embed_pe(ids)
    for layer in range(cfg.num_encoder_layers):
        x = parts.encoder_layer(layer, x)
    assert np.isfinite(x).all()
    rng = np.random.default_rng(7)
    for f in range(3):
        xin = (rng.standard_normal((2, cfg.d_model)) * 0.5).astype(np.float32)
        t = whole.temporal_step(xin, f)
        h = xin
        for layer in range(cfg.num_temporal_layers):
            h = parts.decoder_layer(0, layer, f, h)
        np.testing.assert_array_equal(h, t)
        d = t
        for lvl in range(3):
            lg = whole.depth_step(d, lvl)
            g = d
            for layer in range(cfg.num_depth_layers):
                g = parts.decoder_layer(1, layer, lvl, g)
            np.testing.assert_array_equal(parts.lm_head(g, 0, cfg.vocab_size), lg)
            lo = cfg.codec_offset + lvl * cfg.codebook_size
            np.testing.assert_array_equal(parts.lm_head(g, lo, lo + cfg.codebook_size),
                                          lg[:, lo:lo + cfg.codebook_size])
            d = (rng.standard_normal((2, cfg.d_model)) * 0.5).astype(np.float32)
    K, V = parts.get_cache(0, 1, cfg.max_frames)
    Kw, Vw = whole.get_cache(0, 1, cfg.max_frames)
    np.testing.assert_array_equal(K, Kw)
    np.testing.assert_array_equal(V, Vw)


def test_frame_generation_equals_generate(mrtdf, oracle, tiny_weights):
    """gen_begin + gen_frame (masked: level-slice lm_head) == generate."""
    cfg = mrtdf.preset("tiny", 1)
    ids = random_ids(cfg, 2, cfg.max_encoder_length, seed=8)
    a = oracle.Oracle(tiny_weights, cfg.as_ints())
    b = oracle.Oracle(tiny_weights, cfg.as_ints())
    want = a.generate(ids, cfg.max_frames, 4.0, 1.1, 40, True, 3)
    b.gen_begin(ids)
    got = np.stack([b.gen_frame(f, 4.0, 1.1, 40, True, 3) for f in range(cfg.max_frames)])
    np.testing.assert_array_equal(got, want)

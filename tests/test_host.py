"""CPU-side tests of the C ABI library: it loads, exports every symbol that
include/mrtdf.h declares, and its host logic (presets, weight bundle writer,
streaming glue, error paths) behaves like the reference. No GPU needed."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols(header="mrtdf.h", prefix="mrtdf_"):
    text = open(os.path.join(ROOT, "include", header)).read()
    return sorted(set(re.findall(r"\b(" + prefix + r"[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(mrtdf):
    import mrtss

    lib = mrtdf.lib()
    declared = _declared_symbols()
    assert len(declared) >= 20
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    assert sorted(mrtdf.EXPORTS) == sorted(declared)
    # the SpectroStream decode phase (include/mrtss.h) lives in the same library
    codec = _declared_symbols("mrtss.h", "mrtss_")
    assert len(codec) >= 10
    missing = [s for s in codec if not hasattr(lib, s)]
    assert not missing, missing
    assert sorted(mrtss.EXPORTS) == sorted(codec)
    # the style path (include/mrtmc.h) too
    import mrtmc

    style = _declared_symbols("mrtmc.h", "mrtmc_")
    assert len(style) >= 8
    missing = [s for s in style if not hasattr(lib, s)]
    assert not missing, missing
    assert sorted(mrtmc.EXPORTS) == sorted(style)
    # the C ABI headers, plus the header-only C++ wrapper over mrtdf.h
    assert sorted(os.listdir(os.path.join(ROOT, "include"))) == ["mrtdf.h", "mrtdf.hpp", "mrtmc.h", "mrtss.h"]


def test_version(mrtdf):
    assert b"sm_100a" in mrtdf.lib().mrtdf_version()


def test_presets_match_reference_configs(mrtdf):
    base = mrtdf.preset("base")
    # DepthformerConfig defaults, depthformer/model.h:47-68
    assert (base.vocab_size, base.d_model, base.d_kv, base.d_ff, base.num_heads) == (29824, 768, 64, 2048, 12)
    assert (base.num_encoder_layers, base.num_temporal_layers, base.num_depth_layers) == (12, 20, 4)
    assert (base.max_encoder_length, base.rvq_depth) == (1006, 16)
    assert (base.temporal_num_buckets, base.temporal_max_distance) == (128, 128)
    assert (base.depth_num_buckets, base.depth_max_distance) == (16, 16)
    large = mrtdf.preset("large")  # model.cpp:38-48
    assert (large.d_model, large.d_ff, large.num_heads) == (1024, 2816, 16)
    assert (large.num_encoder_layers, large.num_temporal_layers, large.num_depth_layers) == (24, 40, 8)
    hyb = mrtdf.preset("hybrid")
    assert (hyb.d_model, hyb.num_heads, hyb.d_ff, hyb.vocab_size) == (1024, 16, 2816, 16388)
    assert (hyb.num_encoder_layers, hyb.num_temporal_layers, hyb.num_depth_layers) == (12, 20, 4)
    assert (hyb.temporal_num_buckets, hyb.temporal_max_distance) == (32, 128)
    assert (hyb.codebook_size, hyb.codec_offset, hyb.max_frames) == (1024, 2, 50)
    with pytest.raises(mrtdf.MrtdfError):
        mrtdf.preset("nope")


def test_random_bundle_layout_and_stats(mrtdf, tiny_weights):
    from safetensors.numpy import load_file

    w = load_file(tiny_weights)
    cfg = mrtdf.preset("tiny")
    d, inner, ff, V = cfg.d_model, cfg.inner, cfg.d_ff, cfg.vocab_size
    assert w["token_embedding.weight"].shape == (V, d)
    assert w["lm_head.weight"].shape == (V, d)
    assert w["encoder_layers.0.self_attn.o_proj.weight"].shape == (d, inner)  # Linear is (out, in)
    assert w["temporal_layers.1.cross_attn.k_proj.weight"].shape == (inner, d)
    assert w["depth_layers.0.ffn.wo.weight"].shape == (d, ff)
    assert w["temporal_rel_pos.relative_attention_bias.weight"].shape == (cfg.temporal_num_buckets, cfg.num_heads)
    assert "depth_layers.0.cross_attn.q_proj.weight" not in w
    n_enc = 1 + 9 * cfg.num_encoder_layers + 1
    n_tmp = 1 + 14 * cfg.num_temporal_layers
    n_dep = 1 + 9 * cfg.num_depth_layers + 2
    assert len(w) == n_enc + n_tmp + n_dep
    assert np.all(w["decoder_norm.weight"] == 1.0)
    x = w["temporal_layers.0.ffn.wi_0.weight"].ravel()
    assert abs(x.mean()) < 0.002 and abs(x.std() - 0.02) < 0.001


def test_random_bundle_is_deterministic(mrtdf, tmp_path):
    cfg = mrtdf.preset("tiny")
    a, b, c = (str(tmp_path / n) for n in ("a", "b", "c"))
    mrtdf.write_random_safetensors(cfg, 3, a)
    mrtdf.write_random_safetensors(cfg, 3, b)
    mrtdf.write_random_safetensors(cfg, 4, c)
    assert open(a, "rb").read() == open(b, "rb").read()
    assert open(a, "rb").read() != open(c, "rb").read()


def test_encoder_inputs_empty_context(mrtdf):
    # System::empty_state (system.cpp:165-175): every context slot is -1, so
    # build_encoder_inputs_host (system.cpp:62-95) yields MASK everywhere
    # except the style ids of row 0.
    ctx = -np.ones((250, 16), np.int32)
    style = np.arange(6, dtype=np.int32) + 17410
    out = mrtdf.build_encoder_inputs(ctx, style, 4, 1024, 2)
    assert out.shape == (2, 1006)
    assert np.all(out[0, :1000] == 1) and np.all(out[0, 1000:] == style)
    assert np.all(out[1] == 1)


def test_encoder_inputs_layout(mrtdf):
    rng = np.random.default_rng(0)
    ctx = rng.integers(-1, 1024, size=(250, 16)).astype(np.int32)
    style = rng.integers(0, 5000, size=6).astype(np.int32)
    out = mrtdf.build_encoder_inputs(ctx, style, 4, 1024, 2)
    want = np.where(ctx[:, :4] >= 0, 2 + np.arange(4)[None] * 1024 + ctx[:, :4], 1).reshape(-1)
    np.testing.assert_array_equal(out[0, :1000], want)
    np.testing.assert_array_equal(out[1, :1000], want)
    np.testing.assert_array_equal(out[1, 1000:], np.ones(6, np.int32))


def test_context_roll(mrtdf):
    ctx = np.arange(250 * 16, dtype=np.int32).reshape(250, 16)
    new = -np.arange(50 * 16, dtype=np.int32).reshape(50, 16) - 7
    out = mrtdf.context_roll(ctx, new)
    # system.cpp:320-333: new[f] = old[(f + 50) % 250], last 50 frames = new codes
    want = np.concatenate([ctx[50:], new])
    np.testing.assert_array_equal(out, want)


def test_rvq_llm_round_trip(mrtdf):
    rng = np.random.default_rng(1)
    rvq = rng.integers(0, 1024, size=(50, 16)).astype(np.int32)
    llm = mrtdf.rvq_to_llm(rvq, 1024, 2)
    np.testing.assert_array_equal(llm, 2 + np.arange(16)[None] * 1024 + rvq)
    np.testing.assert_array_equal(mrtdf.llm_to_rvq(llm, 1024, 2), rvq)
    bad = llm.copy()
    bad[3, 5] = 2 + 4 * 1024 + 1  # level-4 code in the level-5 slot
    with pytest.raises(mrtdf.MrtdfError, match="RVQ structure"):
        mrtdf.llm_to_rvq(bad, 1024, 2)


def test_create_fails_cleanly_without_sm100(mrtdf):
    """Without a B200 the engine refuses with a CUDA status instead of
    crashing or falling back to the CPU."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(mrtdf.MrtdfError) as ei:
        mrtdf.Engine(mrtdf.preset("tiny"))
    assert ei.value.code == 2  # MRTDF_ERR_CUDA


def test_unwritable_bundle_path_is_an_io_error(mrtdf, tmp_path):
    lib = mrtdf.lib()
    cfg = mrtdf.preset("tiny")
    rc = lib.mrtdf_write_random_safetensors(ctypes.byref(cfg), 0, ctypes.c_float(0.02), 1,
                                            str(tmp_path / "nodir" / "x").encode())
    assert rc == 3  # MRTDF_ERR_IO
    assert b"cannot write" in lib.mrtdf_last_error()


def test_invalid_config_is_rejected(mrtdf):
    cfg = mrtdf.preset("tiny").replace(d_kv=32)
    with pytest.raises(mrtdf.MrtdfError, match="d_kv"):
        mrtdf.Engine(cfg)


def test_codec_create_fails_cleanly_without_sm100(mrtdf):
    """The SpectroStream decode phase refuses without a B200 too (no CPU
    fallback)."""
    import torch

    import mrtss

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(mrtdf.MrtdfError) as ei:
        mrtss.Codec(max_batch=1, max_frames=4)
    assert ei.value.code == 2  # MRTDF_ERR_CUDA


def test_style_model_fails_cleanly_without_sm100(mrtdf):
    """The style path (include/mrtmc.h) refuses without a B200 (no CPU
    fallback), and rejects bad arguments before touching a device."""
    import torch

    import mrtmc

    lib = mrtmc.lib()
    out = ctypes.c_void_p()
    assert lib.mrtmc_create(0, 0, ctypes.byref(out)) == 1  # max_batch must be in [1, 64]
    assert lib.mrtmc_create(0, 65, ctypes.byref(out)) == 1
    assert lib.mrtmc_create(0, 1, None) == 1
    assert lib.mrtmc_embed_text(None, None, None, 1, 1, None) == 1  # NULL model
    assert lib.mrtmc_embed_kernels(None, 1, 1) == -1
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(mrtdf.MrtdfError) as ei:
        mrtmc.StyleModel(max_batch=1)
    assert ei.value.code == 2  # MRTDF_ERR_CUDA


def test_codec_writer_argument_errors(mrtdf, tmp_path):
    import mrtss

    lib = mrtss.lib()
    ok_dec, ok_cb = str(tmp_path / "d.safetensors").encode(), str(tmp_path / "c.safetensors").encode()
    assert lib.mrtss_write_random_safetensors(0, 0, ok_dec, ok_cb) == 1  # levels must be positive
    assert lib.mrtss_write_random_safetensors(0, 16, None, ok_cb) == 1
    rc = lib.mrtss_write_random_safetensors(0, 16, str(tmp_path / "nodir" / "d").encode(), ok_cb)
    assert rc == 3 and b"cannot write" in lib.mrtdf_last_error()  # MRTDF_ERR_IO
    # the codebook bundle holds "codebooks" (levels, 1024, 256)
    assert lib.mrtss_write_random_safetensors(0, 4, ok_dec, ok_cb) == 0
    from safetensors.numpy import load_file

    assert load_file(ok_cb.decode())["codebooks"].shape == (4, 1024, 256)
    # the same seed writes the same bundle
    again = str(tmp_path / "d2.safetensors").encode()
    assert lib.mrtss_write_random_safetensors(0, 4, again, str(tmp_path / "c2.safetensors").encode()) == 0
    assert open(ok_dec, "rb").read() == open(again, "rb").read()


# ---------------------------------------------------------------------------
# resolve_inference_bundle (weights.cpp:72-120)
# ---------------------------------------------------------------------------
BUNDLE_FILES = {
    "spectrostream_encoder": "spectrostream_encoder.safetensors",
    "spectrostream_decoder": "spectrostream_decoder.safetensors",
    "spectrostream_codebooks": "spectrostream_codebooks.safetensors",
    "musiccoca_encoder": "musiccoca_encoder.safetensors",
    "musiccoca_codebooks": "musiccoca_codebooks.safetensors",
    "musiccoca_vocab": "musiccoca_vocab.model",
}


def _make_bundle(root, tag, skip=()):
    (root / "depthformer").mkdir(parents=True, exist_ok=True)
    for field, name in BUNDLE_FILES.items():
        if field not in skip:
            (root / name).write_bytes(b"x")
    if "depthformer" not in skip:
        (root / "depthformer" / f"depthformer_{tag}.safetensors").write_bytes(b"x")


@pytest.mark.parametrize("tag", ["base", "large"])
def test_resolve_inference_bundle_paths(mrtdf, tmp_path, tag):
    _make_bundle(tmp_path, tag)
    p = mrtdf.resolve_inference_bundle(str(tmp_path), tag)
    for field, name in BUNDLE_FILES.items():
        assert p[field] == str(tmp_path / name)
    assert p["depthformer"] == str(tmp_path / "depthformer" / f"depthformer_{tag}.safetensors")


def test_resolve_inference_bundle_errors(mrtdf, tmp_path):
    ERR_IO = 3
    # not a directory (a file, and a missing path)
    f = tmp_path / "file"
    f.write_bytes(b"x")
    for root in (f, tmp_path / "missing"):
        with pytest.raises(mrtdf.MrtdfError) as e:
            mrtdf.resolve_inference_bundle(str(root), "base")
        assert e.value.code == ERR_IO and "not a directory" in str(e.value)
    # every missing file is listed (the other checkpoint's tag is missing too)
    root = tmp_path / "cache"
    _make_bundle(root, "base", skip=("musiccoca_vocab", "spectrostream_codebooks"))
    with pytest.raises(mrtdf.MrtdfError) as e:
        mrtdf.resolve_inference_bundle(str(root), "base")
    msg = str(e.value)
    assert e.value.code == ERR_IO and "Incomplete Magenta RT C++ inference bundle" in msg
    assert "MusicCoCa SentencePiece vocab" in msg and "SpectroStream codebooks" in msg
    assert "SpectroStream encoder" not in msg
    with pytest.raises(mrtdf.MrtdfError) as e:
        mrtdf.resolve_inference_bundle(str(root), "large")
    assert "depthformer_large.safetensors" in str(e.value)

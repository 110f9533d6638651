"""The style path on the GPU (include/mrtmc.h: MusicCoCa text tower +
style RVQ, float32) against the float32 CPU oracle
(oracle/musiccoca_oracle.cpp) on a random-init bundle with the reference's
key layout.

Tolerance: embeddings within 1e-4 of the largest |value| (the bound the
oracle itself meets against an independent torch formulation; both sides
compute in float32 and differ only in summation order). Style tokens: equal
(the argmin over 1024 random codewords has no near-ties at these sizes)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import STYLE_LEVELS, STYLE_VOCAB, style_prompt

pytestmark = pytest.mark.gpu

ERR_INVALID, ERR_STATE, ERR_KEY, ERR_RANGE = 1, 4, 5, 7


@pytest.fixture(scope="module")
def models(mrtdf, oracle, style_bundle):
    import mrtmc

    enc, cb, _ = style_bundle
    gpu = mrtmc.StyleModel(max_batch=4).load_safetensors(enc, cb)
    orc = oracle.StyleOracle(enc, cb)
    yield gpu, orc
    orc.close()
    gpu.close()


def _batch(pieces, seed):
    rng = np.random.default_rng(seed)
    ids, pad = zip(*(style_prompt(rng, n) for n in pieces))
    return np.concatenate(ids), np.concatenate(pad)


def _close(got, want):
    err = np.abs(got - want).max()
    assert err <= 1e-4 * np.abs(want).max(), (err, np.abs(want).max())
    return err


@pytest.mark.parametrize("L", [128, 48, 1])
def test_embed_text_matches_oracle(models, L):
    gpu, orc = models
    ids, pad = _batch([0, 3, 40, 127][: 4], seed=L)
    ids, pad = ids[:, :L], pad[:, :L]
    got = gpu.embed_text(ids, pad)
    want = orc.embed_text(ids, pad)
    assert got.shape == (4, 768) and np.isfinite(got).all()
    print(f"L = {L}: max |gpu - oracle| = {_close(got, want):.3e} (max |value| {np.abs(want).max():.3f})")
    # one prompt alone (another split-K plan for M = L rows) agrees too
    _close(gpu.embed_text(ids[2:3], pad[2:3]), want[2:3])


def test_embed_text_is_deterministic(models):
    gpu, _ = models
    ids, pad = _batch([5, 60], seed=3)
    a = gpu.embed_text(ids, pad)
    b = gpu.embed_text(ids, pad)
    np.testing.assert_array_equal(a, b)


def test_quantize_matches_oracle(models):
    gpu, orc = models
    ids, pad = _batch([2, 17, 90, 127], seed=9)
    emb = orc.embed_text(ids, pad)
    rand = (np.random.default_rng(4).standard_normal((60, 768)) * 0.5).astype(np.float32)
    x = np.concatenate([emb, rand])
    np.testing.assert_array_equal(gpu.quantize(x, STYLE_LEVELS), orc.quantize(x, STYLE_LEVELS))
    np.testing.assert_array_equal(gpu.quantize(x[:5], 3), orc.quantize(x[:5], 3))


def test_style_tokens_lm(models, mrtdf):
    """StyleModel::style_tokens_lm (style_model.cpp:111-122): the first 6 RVQ
    levels of the prompt's embedding as LLM ids at the style offset
    2 + 16 * 1024 + 1024 (system.h:80-82)."""
    gpu, orc = models
    ids, pad = _batch([12, 33], seed=5)
    got = gpu.style_tokens_lm(ids, pad, 6, 1024, 17410)
    want = mrtdf.rvq_to_llm(orc.quantize(orc.embed_text(ids, pad), STYLE_LEVELS)[:, :6], 1024, 17410)
    np.testing.assert_array_equal(got, want)
    assert got.min() >= 17410 and got.max() < 17410 + 6 * 1024


def test_launch_plan(models):
    gpu, _ = models
    # embedding + 12 x (2 LayerNorms, attention, 4 GEMMs) + 2 LayerNorms +
    # pooler k|v GEMM, attention, o_proj GEMM, plus one epilogue launch per
    # split-K GEMM
    n = gpu.embed_kernels(1, 128)
    assert 1 + 12 * 7 + 2 + 3 <= n <= 1 + 12 * 11 + 2 + 5, n


def test_errors(models, mrtdf, style_bundle, tmp_path):
    import mrtmc
    from safetensors.numpy import save_file

    gpu, _ = models
    ids, pad = _batch([4], seed=1)
    bad = ids.copy()
    bad[0, 2] = STYLE_VOCAB
    for args, code in [((bad, pad), ERR_RANGE),
                       ((np.zeros((1, 129), np.int32), np.zeros((1, 129), np.float32)), ERR_RANGE),
                       ((np.zeros((5, 8), np.int32), np.zeros((5, 8), np.float32)), ERR_RANGE)]:
        with pytest.raises(mrtdf.MrtdfError) as e:
            gpu.embed_text(*args)
        assert e.value.code == code, e.value
    with pytest.raises(mrtdf.MrtdfError) as e:
        gpu.quantize(np.zeros((2, 768), np.float32), STYLE_LEVELS + 1)
    assert e.value.code == ERR_INVALID
    # still usable after the errors
    assert np.isfinite(gpu.embed_text(ids, pad)).all()
    # a second load into the same model, and a bundle without a key
    enc, cb, w = style_bundle
    with pytest.raises(mrtdf.MrtdfError) as e:
        gpu.load_safetensors(enc, cb)
    assert e.value.code == ERR_STATE
    part = {k: v for k, v in w.items() if k != "text_layers.7.ffn_w2.bias"}
    path = str(tmp_path / "partial.safetensors")
    save_file(part, path)
    m = mrtmc.StyleModel(max_batch=1)
    with pytest.raises(mrtdf.MrtdfError) as e:
        m.load_safetensors(path, cb)
    assert e.value.code == ERR_KEY and "text_layers.7.ffn_w2.bias" in str(e.value)
    with pytest.raises(mrtdf.MrtdfError) as e:
        m.embed_text(ids, pad)
    assert e.value.code == ERR_STATE
    m.close()

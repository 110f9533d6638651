"""Committed golden vectors: tests/golden/tiny_golden.npz (made by
tests/golden/make_golden.py from the Depthformer oracle on the tiny config)
and tests/golden/codec_golden.npz (made by tests/golden/make_codec_golden.py
from the SpectroStream oracle).

CPU: the weight generator and the oracle still reproduce them bit for bit.
GPU: the engine matches them within the parity tolerances."""
from __future__ import annotations

import hashlib
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "tiny_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_weight_generator_unchanged(tiny_weights, golden):
    sha = hashlib.sha256(open(tiny_weights, "rb").read()).hexdigest()
    assert sha == str(golden["weights_sha256"])


def test_oracle_reproduces_golden(mrtdf, oracle, tiny_weights, golden):
    from make_golden import make  # tests/golden is on sys.path (conftest)

    data = make(tiny_weights, mrtdf.preset("tiny", mrtdf.DTYPE_FP32), mrtdf.preset("tiny", mrtdf.DTYPE_BF16))
    for k, v in data.items():
        np.testing.assert_array_equal(v, golden[k], err_msg=k)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,key,tol", [(0, "tf_logits_fp32", 1e-4), (1, "tf_logits_bf16", 2e-2)])
def test_engine_teacher_forced_vs_golden(mrtdf, tiny_weights, golden, dtype, key, tol):
    cfg = mrtdf.preset("tiny", dtype)
    eng = mrtdf.Engine(cfg).load_safetensors(tiny_weights)
    got = mrtdf.Stream(eng, 1, True).teacher_forced_logits(golden["ids"], golden["forced"], 1)
    assert np.abs(got - golden[key]).max() <= tol


@pytest.mark.gpu
def test_engine_ids_vs_golden(mrtdf, tiny_weights, golden):
    cfg = mrtdf.preset("tiny", mrtdf.DTYPE_FP32)
    eng = mrtdf.Engine(cfg).load_safetensors(tiny_weights)
    F = cfg.max_frames
    st = mrtdf.Stream(eng, 1, True)
    np.testing.assert_array_equal(st.generate_tokens(golden["ids"], mrtdf.gen_opts(cfg, F, temperature=0.0))[0],
                                  golden["greedy_fp32"])
    np.testing.assert_array_equal(st.generate_tokens(golden["ids"], mrtdf.gen_opts(cfg, F, seed=1))[0],
                                  golden["sampled_fp32_seed1"])
    st1 = mrtdf.Stream(eng, 1, False)
    np.testing.assert_array_equal(
        st1.generate_tokens(golden["ids"][:1], mrtdf.gen_opts(cfg, F, temperature=0.0))[0], golden["greedy_fp32_nocfg"])


# ---- SpectroStream decode phase (tests/golden/codec_golden.npz) -------------
CODEC_GOLDEN = os.path.join(HERE, "golden", "codec_golden.npz")


def test_codec_oracle_reproduces_golden(mrtdf, oracle, tmp_path):
    """The codec weight generator writes the same bundles and the float32
    oracle reproduces the committed outputs (to 1e-6 of each array's largest
    value: libm's exp / cos may pick a different code path per CPU)."""
    import make_codec_golden as mcg

    golden = np.load(CODEC_GOLDEN)
    dec, cb = mcg.bundles(str(tmp_path))
    assert hashlib.sha256(open(dec, "rb").read()).hexdigest() == str(golden["decoder_sha256"])
    assert hashlib.sha256(open(cb, "rb").read()).hexdigest() == str(golden["codebooks_sha256"])
    data = mcg.make(dec, cb)
    np.testing.assert_array_equal(data["codes"], golden["codes"])
    np.testing.assert_array_equal(data["dequant"], golden["dequant"])  # float32 adds in level order
    for k in ("decoded", "audio", "istft"):
        want = golden[k]
        assert data[k].shape == want.shape, k
        assert np.abs(data[k] - want).max() <= 1e-6 * np.abs(want).max(), k

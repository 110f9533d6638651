"""Failure detection on the device, without a GPU fault.

* A bounded device wait runs out: one CTA waits on an mbarrier that nothing
  completes (no copy in flight); the wait gives up after its time bound,
  the call returns MRTDF_ERR_TIMEOUT, and the stream keeps working.
* A draw with no valid candidate (NaN logits) is an error, not a silent
  token: mrtdf_sample returns MRTDF_ERR_INVALID.
"""
from __future__ import annotations

import time

import numpy as np
import pytest

from conftest import random_ids

pytestmark = pytest.mark.gpu

ERR_INVALID = 1
ERR_TIMEOUT = 6


def test_device_wait_timeout_reports_and_recovers(mrtdf, tiny_weights):
    cfg = mrtdf.preset("tiny", mrtdf.DTYPE_BF16)
    eng = mrtdf.Engine(cfg).load_safetensors(tiny_weights)
    st = mrtdf.Stream(eng, 1, True)
    for timeout_us in (1000, 20000):
        t0 = time.perf_counter()
        with pytest.raises(mrtdf.MrtdfError) as e:
            st.check_wait_timeout(timeout_us)
        elapsed = time.perf_counter() - t0
        assert e.value.code == ERR_TIMEOUT, e.value
        assert elapsed < 2.0, elapsed  # the wait ends at its bound, not at the 0.5 s production default
    # the error word was cleared and the stream still decodes
    ids = random_ids(cfg, 2, cfg.max_encoder_length, seed=3)
    toks = st.generate_tokens(ids, mrtdf.gen_opts(cfg, cfg.max_frames, seed=2))
    lo = cfg.codec_offset + np.arange(cfg.rvq_depth) * cfg.codebook_size
    assert np.all((toks[0] >= lo) & (toks[0] < lo + cfg.codebook_size))
    st.sync()
    with pytest.raises(mrtdf.MrtdfError) as e:
        st.check_wait_timeout(0)
    assert e.value.code == 7


@pytest.mark.parametrize("temperature", [0.0, 1.1])
def test_sample_without_candidate_is_an_error(mrtdf, tiny_weights, temperature):
    cfg = mrtdf.preset("tiny", mrtdf.DTYPE_FP32)
    eng = mrtdf.Engine(cfg).load_safetensors(tiny_weights)
    logits = np.full((2, cfg.vocab_size), np.nan, np.float32)
    o = mrtdf.gen_opts(cfg, 1, temperature=temperature, top_k=40, guidance_weight=4.0)
    with pytest.raises(mrtdf.MrtdfError) as e:
        eng.sample(logits, 0, 3, o)
    assert e.value.code == ERR_INVALID
    # finite logits still sample (the engine's device state is unaffected)
    ok = np.random.default_rng(0).standard_normal((2, cfg.vocab_size)).astype(np.float32)
    tok = eng.sample(ok, 0, 3, o)
    lo = cfg.codec_offset + 3 * cfg.codebook_size
    assert lo <= tok < lo + cfg.codebook_size

"""Property tests of the host streaming glue (system.cpp:62-95, 320-333;
rvq.cpp:105-134) over random shapes and values, with numpy restatements of
the reference's arithmetic as the checker. No GPU needed."""
from __future__ import annotations

import numpy as np
import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402

SETTINGS = settings(max_examples=60, deadline=None)


@SETTINGS
@given(frames=st.integers(1, 64), depth=st.integers(1, 16), cb=st.sampled_from([4, 64, 1024]),
       offset=st.integers(0, 5), seed=st.integers(0, 2**31 - 1))
def test_rvq_llm_maps_are_inverse(mrtdf, frames, depth, cb, offset, seed):
    # rvq_to_llm: offset + level * C + code; llm_to_rvq (safe) recovers the code
    rng = np.random.default_rng(seed)
    rvq = rng.integers(0, cb, size=(frames, depth)).astype(np.int32)
    llm = mrtdf.rvq_to_llm(rvq, cb, offset)
    np.testing.assert_array_equal(llm, offset + np.arange(depth)[None] * cb + rvq)
    np.testing.assert_array_equal(mrtdf.llm_to_rvq(llm, cb, offset), rvq)


@SETTINGS
@given(frames=st.integers(1, 16), depth=st.integers(2, 16), cb=st.sampled_from([4, 64, 1024]),
       seed=st.integers(0, 2**31 - 1))
def test_llm_to_rvq_rejects_a_code_of_another_level(mrtdf, frames, depth, cb, seed):
    rng = np.random.default_rng(seed)
    llm = mrtdf.rvq_to_llm(rng.integers(0, cb, size=(frames, depth)).astype(np.int32), cb, 2)
    f, d = rng.integers(0, frames), rng.integers(0, depth)
    other = (d + 1 + rng.integers(0, depth - 1)) % depth  # any level but d
    llm[f, d] = 2 + other * cb + rng.integers(0, cb)
    with pytest.raises(mrtdf.MrtdfError):
        mrtdf.llm_to_rvq(llm, cb, 2)


@SETTINGS
@given(ctx_frames=st.integers(2, 64), depth=st.integers(1, 16), seed=st.integers(0, 2**31 - 1),
       data=st.data())
def test_context_roll_shifts_and_appends(mrtdf, ctx_frames, depth, seed, data):
    new_frames = data.draw(st.integers(1, ctx_frames))
    rng = np.random.default_rng(seed)
    ctx = rng.integers(-1, 1024, size=(ctx_frames, depth)).astype(np.int32)
    new = rng.integers(0, 1024, size=(new_frames, depth)).astype(np.int32)
    out = mrtdf.context_roll(ctx, new)
    np.testing.assert_array_equal(out, np.concatenate([ctx[new_frames:], new]))


@SETTINGS
@given(ctx_frames=st.integers(1, 64), depth=st.integers(4, 16), enc_depth=st.integers(1, 4),
       style_len=st.integers(0, 8), seed=st.integers(0, 2**31 - 1))
def test_encoder_inputs_match_restatement(mrtdf, ctx_frames, depth, enc_depth, style_len, seed):
    # row 0: context levels < enc_depth as offset + level * C + code (MASK = 1
    # where the code is negative), then the style ids; row 1: the same
    # context, style masked (system.cpp:78-93)
    rng = np.random.default_rng(seed)
    ctx = rng.integers(-1, 1024, size=(ctx_frames, depth)).astype(np.int32)
    style = rng.integers(0, 30000, size=style_len).astype(np.int32)
    out = mrtdf.build_encoder_inputs(ctx, style, enc_depth, 1024, 2)
    body = np.where(ctx[:, :enc_depth] >= 0, 2 + np.arange(enc_depth)[None] * 1024 + ctx[:, :enc_depth], 1)
    want0 = np.concatenate([body.reshape(-1), style])
    want1 = np.concatenate([body.reshape(-1), np.ones(style_len, np.int32)])
    np.testing.assert_array_equal(out, np.stack([want0, want1]))

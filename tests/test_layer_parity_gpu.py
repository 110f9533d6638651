"""Layer-by-layer parity of the production kernels at the reference's model
shapes ("hybrid", the benchmark architecture, and the published "base" and
"large" checkpoint shapes) against the CPU oracle, on identical inputs.

Each check feeds ONE production launch sequence (through the engine's probe
entry points: the same kernels, launch shapes and epilogues as a chunk) the
oracle's own bf16 inputs and cache contents, and compares its output with the
oracle's output of that one step:

* one encoder layer at M = 2 x 1006 rows (tcgen05 GEMMs, tensor-core
  attention);
* one temporal layer at cache positions 0, 32 and 49 (self-attention over
  1, 33 and 50 keys inside the q/k/v cluster; cross-attention over 1006
  keys; GEGLU FFN);
* one depth layer at levels 0, 7 and 15;
* lm_head on a level's 1024 rows, and on the whole vocabulary.

Tolerance. Logits: 2e-2 max-abs against the bf16 oracle (BASELINE.json
north_star). Hidden states reach |x| ~ 7 (encoder) and ~ 10 (temporal stack)
on this random-init model, where one bf16 ulp is 0.03 - 0.06, and each layer
chains a dozen bf16 rounding points; when two implementations accumulate in
different fp32 orders some of those roundings go the other way, so no bf16
implementation meets 2e-2 max-abs on every hidden element. For hidden states
the test therefore measures the layer against the fp32 oracle on the same
inputs and requires (a) the engine to be no further from fp32 than the
oracle's own bf16 emulation is (mean and max: the model's bf16 noise floor),
(b) mean |engine - bf16 oracle| within twice that floor, (c) fewer than 1 %
of elements beyond 2e-2 of the bf16 oracle (a decode step has only 2 x 1024
elements, and at |x| >= 4 a single rounding that goes the other way is
already beyond 2e-2) and none beyond 8 bf16 ulps of its value (a wrong
kernel misses all of these by orders of magnitude).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import random_ids

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
FP32_TOL = 1e-4


def bf16_ulp(v: np.ndarray) -> np.ndarray:
    a = np.maximum(np.abs(v).astype(np.float64), 2.0 ** -126)
    return np.exp2(np.floor(np.log2(a)) - 7)


def check_hidden(got, want16, want32, what: str) -> dict:
    got = got.astype(np.float64)
    e16, e32 = np.abs(got - want16), np.abs(got - want32)
    floor = np.abs(want16.astype(np.float64) - want32)
    stats = {"max16": float(e16.max()), "mean16": float(e16.mean()), "max32": float(e32.max()),
             "mean32": float(e32.mean()), "floor_max": float(floor.max()), "floor_mean": float(floor.mean()),
             "frac_gt_tol": float((e16 > BF16_TOL).mean()), "max_abs_value": float(np.abs(want16).max())}
    stats = {k: round(v, 7) for k, v in stats.items()}
    assert stats["mean32"] <= 1.25 * stats["floor_mean"] + 1e-7, (what, stats)
    assert stats["max32"] <= 1.25 * stats["floor_max"] + BF16_TOL, (what, stats)
    assert stats["mean16"] <= 2.0 * stats["floor_mean"] + 1e-7, (what, stats)
    assert stats["frac_gt_tol"] < 1e-2, (what, stats)
    bound = np.maximum(BF16_TOL, 8 * bf16_ulp(want16))
    worst = np.unravel_index(np.argmax(e16 - bound), e16.shape)
    assert (e16 <= bound).all(), (what, stats, worst, float(got[worst]), float(want16[worst]))
    return stats


def check_logits(got, want16, want32, what: str) -> str:
    err = float(np.abs(got - want16).max())
    floor = float(np.abs(want16 - want32).max())
    assert err <= BF16_TOL, (what, err, floor)
    return f"max {err:.3e} (bf16 oracle vs fp32: {floor:.3e})"


@pytest.fixture(scope="module", params=["hybrid", "base", "large"])
def model(request, mrtdf, oracle):
    cfg = mrtdf.preset(request.param, mrtdf.DTYPE_BF16)
    eng = mrtdf.Engine(cfg).load_random(0)
    orc16 = oracle.Oracle.from_random(cfg.as_ints(), 0)
    orc32 = oracle.Oracle.from_random(mrtdf.preset(request.param, mrtdf.DTYPE_FP32).as_ints(), 0)
    ids = random_ids(cfg, 2, cfg.max_encoder_length, seed=20)
    yield request.param, cfg, eng, orc16, orc32, ids
    orc32.close()
    orc16.close()
    eng.close()


def test_encoder_layers(mrtdf, model):
    name, cfg, eng, orc, orc32, ids = model
    st = mrtdf.Stream(eng, 1, True)
    x = orc.embed_pe(ids)
    probe = {0, cfg.num_encoder_layers // 2, cfg.num_encoder_layers - 1}
    for layer in range(cfg.num_encoder_layers):
        want = orc.encoder_layer(layer, x)
        if layer in probe:
            got = st.probe_encoder_layer(layer, x)
            s = check_hidden(got, want, orc32.encoder_layer(layer, x), f"{name} encoder layer {layer}")
            print(f"{name} encoder layer {layer}: {s}")
        x = want
    st.close()


def test_decoder_layers_and_lm_head(mrtdf, model):
    """Temporal layers at positions 0, 32, 49 (after teacher-forced frames
    filled the oracle's caches), then depth layers and lm_head at levels 0,
    7 and 15 of the last frame."""
    name, cfg, eng, orc, orc32, ids = model
    st = mrtdf.Stream(eng, 1, True)
    orc.encode(ids)
    S, Lt, Ld, T, D = cfg.max_encoder_length, cfg.num_temporal_layers, cfg.num_depth_layers, cfg.max_frames, \
        cfg.rvq_depth
    rng = np.random.default_rng(21)
    t_probe, t_layers = {0, 32, T - 1}, {0, Lt // 2, Lt - 1}
    # temporal inputs: frame-mean embeddings are ~N(0, 0.005)
    xs = [(rng.standard_normal((2, cfg.d_model)) * 0.005).astype(np.float32) for _ in range(T)]
    for f in range(T):
        if f in t_probe:
            h = xs[f]
            for layer in range(Lt):
                if layer in t_layers:
                    K, V = orc.get_cache(0, layer, T)
                    Kc, Vc = orc.get_cache(2, layer, S)
                    st.probe_set_cache(2, layer, Kc, Vc)
                    st.probe_set_cache(0, layer, K[:, :, :f], V[:, :, :f])
                    orc32.set_cache(2, layer, Kc, Vc, S)
                    orc32.set_cache(0, layer, K, V, S)
                    want32 = orc32.decoder_layer(0, layer, f, h)
                    got = st.probe_decoder_layer(0, layer, f, h)
                    want = orc.decoder_layer(0, layer, f, h)
                    s = check_hidden(got, want, want32, f"{name} temporal layer {layer} pos {f}")
                    print(f"{name} temporal layer {layer} pos {f}: {s}")
                else:
                    want = orc.decoder_layer(0, layer, f, h)
                h = want
        tout = orc.temporal_step(xs[f], f)  # advances the oracle's frame counter
    # depth stack of the last frame
    d_probe, d_layers = {0, 7, D - 1}, {0, Ld - 1}
    d = tout
    for lvl in range(D):
        if lvl in d_probe:
            g = d
            for layer in range(Ld):
                if layer in d_layers:
                    K, V = orc.get_cache(1, layer, D)
                    st.probe_set_cache(1, layer, K[:, :, :lvl], V[:, :, :lvl])
                    orc32.set_cache(1, layer, K, V, S)
                    want32 = orc32.decoder_layer(1, layer, lvl, g)
                    got = st.probe_decoder_layer(1, layer, lvl, g)
                    want = orc.decoder_layer(1, layer, lvl, g)
                    s = check_hidden(got, want, want32, f"{name} depth layer {layer} level {lvl}")
                    print(f"{name} depth layer {layer} level {lvl}: {s}")
                else:
                    want = orc.decoder_layer(1, layer, lvl, g)
                g = want
            lo = cfg.codec_offset + lvl * cfg.codebook_size
            msg = check_logits(st.probe_lm_head(lvl, g), orc.lm_head(g, lo, lo + cfg.codebook_size),
                               orc32.lm_head(g, lo, lo + cfg.codebook_size), f"{name} lm_head level {lvl}")
            print(f"{name} lm_head level {lvl}: {msg}")
            if lvl == D - 1:
                msg = check_logits(st.probe_lm_head(-1, g), orc.lm_head(g, 0, cfg.vocab_size),
                                   orc32.lm_head(g, 0, cfg.vocab_size), f"{name} lm_head all rows")
                print(f"{name} lm_head all {cfg.vocab_size} rows: {msg}")
        orc.depth_step(d, lvl)  # advances the oracle's depth counter
        d = (rng.standard_normal((2, cfg.d_model)) * 0.02).astype(np.float32)
    st.close()


# ---------------------------------------------------------------------------
# one whole 2 s chunk, fp32, batch 1, greedy, no CFG
# ---------------------------------------------------------------------------
def test_config1_full_chunk_greedy_bit_exact_fp32(mrtdf, oracle):
    cfg = mrtdf.preset("hybrid", mrtdf.DTYPE_FP32)
    eng = mrtdf.Engine(cfg).load_random(0)
    orc = oracle.Oracle.from_random(cfg.as_ints(), 0)
    ids = np.random.default_rng(0).integers(0, cfg.vocab_size, size=(1, cfg.max_encoder_length)).astype(np.int32)
    st = mrtdf.Stream(eng, 1, False)
    o = mrtdf.gen_opts(cfg, 50, temperature=0.0, top_k=40, guidance_weight=0.0)
    got = st.generate_tokens(ids, o)[0]
    want = orc.generate(ids, 50, 0.0, 0.0, 40, True, 0)
    assert got.shape == (50, cfg.rvq_depth)
    np.testing.assert_array_equal(got, want)
    st.close()
    orc.close()
    eng.close()


def test_hybrid_bf16_teacher_forced_50_frames(mrtdf, oracle):
    """A whole chunk of teacher-forced bf16 logits (CFG pair) against the bf16
    and fp32 oracles: per-frame max / mean abs distribution printed; the
    engine is no further from the fp32 logits than the oracle's own bf16
    emulation (the model's bf16 noise floor) and close to the bf16 oracle."""
    cfg = mrtdf.preset("hybrid", mrtdf.DTYPE_BF16)
    eng = mrtdf.Engine(cfg).load_random(0)
    F = 50
    ids = random_ids(cfg, 2, cfg.max_encoder_length, seed=20)
    rng = np.random.default_rng(21)
    toks = np.stack([cfg.codec_offset + np.arange(cfg.rvq_depth) * cfg.codebook_size
                     + rng.integers(0, cfg.codebook_size, cfg.rvq_depth) for _ in range(F)]).astype(np.int32)
    got = mrtdf.Stream(eng, 1, True).teacher_forced_logits(ids, toks, F)
    o16 = oracle.Oracle.from_random(cfg.as_ints(), 0)
    want16 = o16.teacher_forced(ids, toks, F)
    o16.close()
    o32 = oracle.Oracle.from_random(mrtdf.preset("hybrid", 0).as_ints(), 0)
    want32 = o32.teacher_forced(ids, toks, F)
    o32.close()
    e16 = np.abs(got - want16).reshape(F, -1)
    e32 = np.abs(got - want32).reshape(F, -1)
    floor = np.abs(want16 - want32).reshape(F, -1)
    for f in range(0, F, 7):
        print(f"frame {f}: vs bf16 oracle max {e16[f].max():.3e} mean {e16[f].mean():.2e}; "
              f"vs fp32 max {e32[f].max():.3e} mean {e32[f].mean():.2e}; floor max {floor[f].max():.3e}")
    print(f"all frames: vs bf16 max {e16.max():.3e} mean {e16.mean():.2e}; vs fp32 mean {e32.mean():.2e}; "
          f"floor mean {floor.mean():.2e}")
    assert e32.mean() <= 1.25 * floor.mean()
    assert e16.mean() <= 2.0 * floor.mean()
    assert e32.max() <= 1.25 * floor.max() + BF16_TOL


def test_encoder_attention_wide_logits(mrtdf, oracle):
    """Encoder layer 0 with weights N(0, 0.04^2): attention logits of std
    ~12.5, so that the one-pass softmax raises its running maximum mid-row
    (a key tile beats it by more than e^8 and O and the sum are rescaled in
    TMEM) in ~72 % of the (row, head, query, key half) sequences, against
    ~7 % at the N(0, 0.02^2) weights of the tests above (counted on the host
    from the weights under the kernel's tile schedule).

    Hidden values reach |x| ~ 14 here and the attention is peaky, so the
    bf16 emulation itself leaves the fp32 result by more than 2e-2 in more
    than half of the elements (max 0.27); the test requires the engine to be
    no noisier than that: mean / max distance to fp32 within the floor's,
    and its distance to the bf16 oracle (mean, max, share beyond 2e-2) below
    the floor's. A wrong rescale (O kept at the old maximum's scale, a race
    with the previous P V) is off by factors up to e^8 and misses all of
    these."""
    std = 0.04
    cfg = mrtdf.preset("hybrid", mrtdf.DTYPE_BF16)
    eng = mrtdf.Engine(cfg).load_random(0, stddev=std)
    orc16 = oracle.Oracle.from_random(cfg.as_ints(), 0, stddev=std)
    orc32 = oracle.Oracle.from_random(mrtdf.preset("hybrid", mrtdf.DTYPE_FP32).as_ints(), 0, stddev=std)
    ids = random_ids(cfg, 2, cfg.max_encoder_length, seed=20)
    st = mrtdf.Stream(eng, 1, True)
    x = orc16.embed_pe(ids)
    got = st.probe_encoder_layer(0, x).astype(np.float64)
    want16 = orc16.encoder_layer(0, x).astype(np.float64)
    want32 = orc32.encoder_layer(0, x).astype(np.float64)
    e16, e32, floor = np.abs(got - want16), np.abs(got - want32), np.abs(want16 - want32)
    stats = {"max16": e16.max(), "mean16": e16.mean(), "frac16": (e16 > BF16_TOL).mean(), "max32": e32.max(),
             "mean32": e32.mean(), "floor_max": floor.max(), "floor_mean": floor.mean(),
             "floor_frac": (floor > BF16_TOL).mean(), "max_abs_value": np.abs(want16).max()}
    stats = {k: round(float(v), 6) for k, v in stats.items()}
    print(f"hybrid encoder layer 0, weights N(0, {std}^2): {stats}")
    assert stats["mean32"] <= 1.25 * stats["floor_mean"], stats
    assert stats["max32"] <= 1.25 * stats["floor_max"] + BF16_TOL, stats
    assert stats["mean16"] <= stats["floor_mean"], stats
    assert stats["max16"] <= stats["floor_max"], stats
    assert stats["frac16"] <= stats["floor_frac"], stats
    st.close()
    orc32.close()
    orc16.close()
    eng.close()

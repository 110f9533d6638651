"""Parity of the CUDA engine (through the C ABI) against the CPU oracle.

Tolerances: teacher-forced logits within 1e-4 max-abs
in fp32 and 2e-2 in bf16; greedy ids bit-exact in fp32; sampled ids
bit-exact given identical logits and draws.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import random_ids

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-4
BF16_TOL = 2e-2


def _engine(mrtdf, path, name, dtype):
    cfg = mrtdf.preset(name, dtype)
    return cfg, mrtdf.Engine(cfg).load_safetensors(path)


def _forced_tokens(cfg, F, seed):
    rng = np.random.default_rng(seed)
    return np.stack([cfg.codec_offset + np.arange(cfg.rvq_depth) * cfg.codebook_size
                     + rng.integers(0, cfg.codebook_size, cfg.rvq_depth) for _ in range(F)]).astype(np.int32)


# ---------------------------------------------------------------------------
# tiny config: every path, both dtypes
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,tol", [(0, FP32_TOL), (1, BF16_TOL)])
def test_encode_matches_oracle(mrtdf, oracle, tiny_weights, dtype, tol):
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", dtype)
    ids = random_ids(cfg, 2, cfg.max_encoder_length, seed=1)
    st = mrtdf.Stream(eng, 1, True)
    got = st.encode(ids, want_output=True)
    want = oracle.Oracle(tiny_weights, cfg.as_ints()).encode(ids)
    assert np.abs(got - want).max() <= tol


@pytest.mark.parametrize("dtype,tol", [(0, FP32_TOL), (1, BF16_TOL)])
def test_step_api_matches_oracle(mrtdf, oracle, tiny_weights, dtype, tol):
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", dtype)
    ids = random_ids(cfg, 2, 60, seed=2)
    st = mrtdf.Stream(eng, 1, True)
    orc = oracle.Oracle(tiny_weights, cfg.as_ints())
    st.encode(ids)
    orc.encode(ids)
    rng = np.random.default_rng(0)
    x = None
    for f in range(3):
        a = st.temporal_step(x, f)
        b = orc.temporal_step(x, f)
        assert np.abs(a - b).max() <= tol * 4, f
        d = None
        for l in range(4):
            la = st.depth_step(d, l)
            lb = orc.depth_step(d, l)
            assert np.abs(la - lb).max() <= tol, (f, l)
            d = rng.standard_normal((2, cfg.d_model)).astype(np.float32) * 0.5
        x = rng.standard_normal((2, cfg.d_model)).astype(np.float32) * 0.5


@pytest.mark.parametrize("dtype,tol", [(0, FP32_TOL), (1, BF16_TOL)])
@pytest.mark.parametrize("cfg_rows", [1, 2])
def test_teacher_forced_logits(mrtdf, oracle, tiny_weights, dtype, tol, cfg_rows):
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", dtype)
    F = 4
    ids = random_ids(cfg, cfg_rows, cfg.max_encoder_length, seed=3)
    toks = _forced_tokens(cfg, F, seed=4)
    st = mrtdf.Stream(eng, 1, cfg_rows == 2)
    got = st.teacher_forced_logits(ids, toks, F)
    want = oracle.Oracle(tiny_weights, cfg.as_ints()).teacher_forced(ids, toks, F)
    err = np.abs(got - want).max()
    assert err <= tol, err


def test_greedy_ids_bit_exact_fp32(mrtdf, oracle, tiny_weights):
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", 0)
    F = cfg.max_frames
    for rows, seed in [(1, 5), (2, 6)]:
        ids = random_ids(cfg, rows, cfg.max_encoder_length, seed=seed)
        st = mrtdf.Stream(eng, 1, rows == 2)
        o = mrtdf.gen_opts(cfg, F, temperature=0.0, top_k=40, guidance_weight=4.0)
        got = st.generate_tokens(ids, o)[0]
        want = oracle.Oracle(tiny_weights, cfg.as_ints()).generate(ids, F, 4.0, 0.0, 40, True, 0)
        np.testing.assert_array_equal(got, want)


def test_sampled_ids_with_injected_draws_fp32(mrtdf, oracle, tiny_weights):
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", 0)
    F = cfg.max_frames
    ids = random_ids(cfg, 2, cfg.max_encoder_length, seed=7)
    u = np.random.default_rng(8).uniform(1e-7, 1 - 1e-7, (F * cfg.rvq_depth, cfg.vocab_size)).astype(np.float32)
    st = mrtdf.Stream(eng, 1, True)
    o = mrtdf.gen_opts(cfg, F, temperature=1.1, top_k=40, guidance_weight=4.0, uniforms=u)
    got = st.generate_tokens(ids, o)[0]
    want = oracle.Oracle(tiny_weights, cfg.as_ints()).generate(ids, F, 4.0, 1.1, 40, True, 0, uniforms=u)
    np.testing.assert_array_equal(got, want)


def test_sampled_ids_with_philox_fp32(mrtdf, oracle, tiny_weights):
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", 0)
    F = cfg.max_frames
    ids = random_ids(cfg, 2, cfg.max_encoder_length, seed=9)
    st = mrtdf.Stream(eng, 1, True)
    o = mrtdf.gen_opts(cfg, F, temperature=1.1, top_k=40, guidance_weight=4.0, seed=1)
    got = st.generate_tokens(ids, o)[0]
    want = oracle.Oracle(tiny_weights, cfg.as_ints()).generate(ids, F, 4.0, 1.1, 40, True, 1)
    np.testing.assert_array_equal(got, want)


def test_sampler_bit_exact(mrtdf, oracle, tiny_weights):
    """mrtdf_sample == oracle sampler on identical logits and draws."""
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", 0)
    rng = np.random.default_rng(10)
    V = cfg.vocab_size
    for trial in range(120):
        rows = 1 + trial % 2
        logits = rng.standard_normal((rows, V)).astype(np.float32) * 3
        if trial % 3 == 0:
            logits = np.round(logits * 2) / 2  # many ties at the top-k threshold
        T = [0.0, 1.1, 0.5, 2.0][trial % 4]
        k = [40, 1, 0, 64, 7][trial % 5]
        masked = trial % 7 != 0
        level = trial % cfg.rvq_depth
        u = rng.uniform(1e-7, 1 - 1e-7, V).astype(np.float32)
        o = mrtdf.gen_opts(cfg, 1, temperature=T, top_k=k, guidance_weight=4.0, use_vocab_masks=masked)
        got = eng.sample(logits, 0, level, o, uniforms=u)
        want = oracle.sample(logits, level, masked, cfg.codebook_size, cfg.codec_offset, 4.0, T, k, u)
        assert got == want, (trial, got, want)


def test_sampler_philox_draws_match(mrtdf, oracle, tiny_weights):
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", 0)
    rng = np.random.default_rng(11)
    V = cfg.vocab_size
    for trial in range(40):
        logits = rng.standard_normal((2, V)).astype(np.float32)
        frame, level, seed = trial % 5, trial % 16, 1000 + trial
        u = np.array([oracle.philox_uniform(seed, frame * cfg.rvq_depth + level, i) for i in range(V)], np.float32)
        o = mrtdf.gen_opts(cfg, 1, temperature=1.1, top_k=40, guidance_weight=4.0, seed=seed)
        got = eng.sample(logits, frame, level, o, uniforms=None)
        want = oracle.sample(logits, level, True, cfg.codebook_size, cfg.codec_offset, 4.0, 1.1, 40, u)
        assert got == want


def test_graph_replay_equals_stream_launches(mrtdf, tiny_weights):
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", 1)
    ids = random_ids(cfg, 2, cfg.max_encoder_length, seed=12)
    o = mrtdf.gen_opts(cfg, cfg.max_frames, seed=3)
    st = mrtdf.Stream(eng, 1, True)
    a = st.generate_tokens(ids, o)
    b = st.generate_tokens(ids, o)  # graph replay
    os.environ["MRTDF_GRAPH"] = "0"
    try:
        c = st.generate_tokens(ids, o)
    finally:
        del os.environ["MRTDF_GRAPH"]
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(a, c)
    o2 = mrtdf.gen_opts(cfg, cfg.max_frames, seed=4)
    assert not np.array_equal(a, st.generate_tokens(ids, o2))


def test_multi_sequence_stream_equals_single(mrtdf, tiny_weights):
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", 1)
    F = cfg.max_frames
    ids_a = random_ids(cfg, 2, cfg.max_encoder_length, seed=13)
    ids_b = random_ids(cfg, 2, cfg.max_encoder_length, seed=14)
    o = mrtdf.gen_opts(cfg, F)
    multi = mrtdf.Stream(eng, 2, True).generate_tokens(np.concatenate([ids_a, ids_b]), o, seeds=[100, 101])
    single = mrtdf.Stream(eng, 1, True)
    np.testing.assert_array_equal(multi[0], single.generate_tokens(ids_a, o, seeds=[100])[0])
    np.testing.assert_array_equal(multi[1], single.generate_tokens(ids_b, o, seeds=[101])[0])


def test_call_order_errors(mrtdf, tiny_weights):
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", 1)
    st = mrtdf.Stream(eng, 1, True)
    with pytest.raises(mrtdf.MrtdfError) as e:
        st.temporal_step(None, 0)
    assert e.value.code == 4  # MRTDF_ERR_STATE: no cross-attention cache yet
    st.encode(random_ids(cfg, 2, 20, seed=1))
    with pytest.raises(mrtdf.MrtdfError) as e:
        st.temporal_step(None, 1)
    assert e.value.code == 4  # cache size mismatch (model.cpp:326-328)
    st.temporal_step(None, 0)
    with pytest.raises(mrtdf.MrtdfError) as e:
        st.depth_step(None, cfg.rvq_depth)
    assert e.value.code == 7  # MRTDF_ERR_RANGE
    with pytest.raises(mrtdf.MrtdfError) as e:
        st.encode(random_ids(cfg, 2, cfg.max_encoder_length + 1, seed=1))
    assert e.value.code == 7  # seq_len exceeds max_encoder_length (model.cpp:216-218)
    bad = random_ids(cfg, 2, 20, seed=1)
    bad[0, 3] = cfg.vocab_size
    with pytest.raises(mrtdf.MrtdfError) as e:
        st.encode(bad)
    assert e.value.code == 1


# ---------------------------------------------------------------------------
# benchmark architecture (hybrid: d 1024, 12/20/4 layers, vocab 16388)
# ---------------------------------------------------------------------------
def test_hybrid_bf16_teacher_forced(mrtdf, oracle, hybrid_weights):
    """Full-size bf16 logits against the fp32 oracle, measured against the
    model's own bf16 noise floor.

    On this random-init model two independent bf16 evaluations (the oracle's
    bf16 emulation and the engine) each land about 0.16 max-abs from the
    fp32 logits: fp32 accumulation-order differences flip bf16 roundings and
    the 36 attention layers amplify them. The 2e-2 bf16 bound is therefore
    checked on the tiny config (test_teacher_forced_logits); here the engine
    must be as close to fp32 as the oracle's own bf16 emulation is, and the
    exact algorithm is pinned by the fp32 test below (1e-4)."""
    cfg, eng = _engine(mrtdf, hybrid_weights, "hybrid", 1)
    F = 2
    ids = random_ids(cfg, 2, 1006, seed=20)
    toks = _forced_tokens(cfg, F, seed=21)
    got = mrtdf.Stream(eng, 1, True).teacher_forced_logits(ids, toks, F)
    orc16 = oracle.Oracle(hybrid_weights, cfg.as_ints()).teacher_forced(ids, toks, F)
    orc32 = oracle.Oracle(hybrid_weights, mrtdf.preset("hybrid", 0).as_ints()).teacher_forced(ids, toks, F)
    floor_max = np.abs(orc16 - orc32).max()
    floor_mean = np.abs(orc16 - orc32).mean()
    assert np.abs(got - orc32).max() <= 1.25 * floor_max + BF16_TOL
    assert np.abs(got - orc32).mean() <= 1.25 * floor_mean
    assert np.abs(got - orc16).mean() <= 2.0 * floor_mean


def test_hybrid_fp32_teacher_forced_and_greedy(mrtdf, oracle, hybrid_weights):
    cfg, eng = _engine(mrtdf, hybrid_weights, "hybrid", 0)
    F = 2
    ids = random_ids(cfg, 1, 1006, seed=0)
    orc = oracle.Oracle(hybrid_weights, cfg.as_ints())
    st = mrtdf.Stream(eng, 1, False)
    toks = _forced_tokens(cfg, F, seed=22)
    err = np.abs(st.teacher_forced_logits(ids, toks, F) - orc.teacher_forced(ids, toks, F)).max()
    assert err <= FP32_TOL, err
    o = mrtdf.gen_opts(cfg, F, temperature=0.0)
    np.testing.assert_array_equal(st.generate_tokens(ids, o)[0], orc.generate(ids, F, 0.0, 0.0, 40, True, 0))


def test_hybrid_bf16_chunk_properties(mrtdf, hybrid_weights):
    """A full 50-frame chunk: ids in their level ranges, deterministic, seed-dependent."""
    cfg, eng = _engine(mrtdf, hybrid_weights, "hybrid", 1)
    ids = random_ids(cfg, 2, 1006, seed=23)
    st = mrtdf.Stream(eng, 1, True)
    o = mrtdf.gen_opts(cfg, 50, seed=1)
    a = st.generate_tokens(ids, o)[0]
    b = st.generate_tokens(ids, o)[0]
    np.testing.assert_array_equal(a, b)
    lo = cfg.codec_offset + np.arange(16) * cfg.codebook_size
    assert np.all((a >= lo[None]) & (a < lo[None] + cfg.codebook_size))
    rvq = mrtdf.llm_to_rvq(a, cfg.codebook_size, cfg.codec_offset)
    assert rvq.min() >= 0 and rvq.max() < 1024
    c = st.generate_tokens(ids, mrtdf.gen_opts(cfg, 50, seed=2))[0]
    assert (a != c).mean() > 0.5


# ---------------------------------------------------------------------------
# bf16 self-attention inside the q/k/v cluster vs the separate kernel
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name", ["tiny", "hybrid"])
def test_cluster_self_attention_matches_separate_kernel(mrtdf, tiny_weights, name):
    """Streams of 3 - 8 bf16 rows run one launch per projection; their
    self-attention runs inside the q/k/v launch (one thread-block cluster per
    head) with the separate attention kernel's arithmetic
    (MRTDF_CLUSTER_ATTN=0): bit-identical step outputs and tokens."""
    cfg = mrtdf.preset(name, 1)
    frames = cfg.max_frames if name == "tiny" else 3
    seq = cfg.max_encoder_length if name == "tiny" else 256

    def make():
        e = mrtdf.Engine(cfg)
        return e.load_safetensors(tiny_weights) if name == "tiny" else e.load_random(0)

    outs = []
    for cluster in ("1", "0"):
        old = os.environ.get("MRTDF_CLUSTER_ATTN")
        os.environ["MRTDF_CLUSTER_ATTN"] = cluster
        try:
            eng = make()
        finally:
            if old is None:
                del os.environ["MRTDF_CLUSTER_ATTN"]
            else:
                os.environ["MRTDF_CLUSTER_ATTN"] = old
        st = mrtdf.Stream(eng, 2, True)  # 4 rows
        ids = np.concatenate([random_ids(cfg, 2, seq, seed=21), random_ids(cfg, 2, seq, seed=22)])
        st.encode(ids)
        t = st.temporal_step(None, 0)
        lg = st.depth_step(None, 0)
        gen = st.generate_tokens(ids, mrtdf.gen_opts(cfg, frames, seed=4), seeds=[4, 5])
        outs.append((t, lg, gen))
        st.close()
        eng.close()
    for a, b in zip(outs[0], outs[1]):
        np.testing.assert_array_equal(a, b)


def test_measurement_hooks(mrtdf, tiny_weights):
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", 1)
    ms, flops = eng.bench_encoder(3, cfg.max_encoder_length, 2)
    S, M, d, inn, ff = cfg.max_encoder_length, 3 * cfg.max_encoder_length, cfg.d_model, cfg.inner, cfg.d_ff
    lin = 2 * M * (d * 3 * inn + inn * d + d * 2 * ff + ff * d)
    att = 4 * 3 * cfg.num_heads * S * S * 64
    assert ms > 0 and flops == pytest.approx(cfg.num_encoder_layers * (lin + att)
                                             + 2 * M * d * 2 * cfg.num_temporal_layers * inn)
    st = mrtdf.Stream(eng, 1, True)
    o = mrtdf.gen_opts(cfg, cfg.max_frames, seed=3)
    us, b, n = st.bench_depth(o, cfg.max_frames, 2)
    # one CFG pair in bf16: (self phase, FFN phase) x layers + lm_head + sampler
    assert us > 0 and b > 0 and n == cfg.num_depth_layers * 2 + 2
    st.sync()


def test_device_streaming_equals_host_loop(mrtdf, tiny_weights):
    """mrtdf_generate_stream_dev == the host System loop (encoder ids ->
    generate_tokens -> llm_to_rvq -> context roll), chunk by chunk."""
    torch = pytest.importorskip("torch")
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", 1)
    nseq, K, F, enc_depth, style_depth = 2, 3, cfg.max_frames, 4, 6
    ctx_frames = (cfg.max_encoder_length - style_depth) // enc_depth
    rng = np.random.default_rng(31)
    ctx = -np.ones((nseq, ctx_frames, cfg.rvq_depth), np.int32)
    ctx[0, -5:] = rng.integers(0, cfg.codebook_size, (5, cfg.rvq_depth))  # a partly filled context
    style = rng.integers(cfg.codec_offset, cfg.codec_offset + cfg.rvq_depth * cfg.codebook_size,
                         (nseq, style_depth)).astype(np.int32)
    seeds = [100 + 10 * k + i for k in range(K) for i in range(nseq)]
    o = mrtdf.gen_opts(cfg, F)
    ctx_dev = torch.from_numpy(ctx.copy()).cuda()
    style_dev = torch.from_numpy(style).cuda()
    out_dev = torch.full((K, nseq, F, cfg.rvq_depth), -1, dtype=torch.int32, device="cuda")
    st_dev = mrtdf.Stream(eng, nseq, True)
    st_dev.generate_stream_dev(ctx_dev.data_ptr(), ctx_frames, enc_depth, style_dev.data_ptr(), style_depth, K, o,
                               out_dev.data_ptr(), seeds=seeds)
    st_dev.sync()
    st = mrtdf.Stream(eng, nseq, True)
    want = []
    for k in range(K):
        ids = np.concatenate([mrtdf.build_encoder_inputs(ctx[i], style[i], enc_depth, cfg.codebook_size,
                                                         cfg.codec_offset) for i in range(nseq)], axis=0)
        toks = st.generate_tokens(ids, o, seeds=seeds[k * nseq:(k + 1) * nseq])
        rvq = np.stack([mrtdf.llm_to_rvq(toks[i], cfg.codebook_size, cfg.codec_offset) for i in range(nseq)])
        ctx = np.stack([mrtdf.context_roll(ctx[i], rvq[i]) for i in range(nseq)])
        want.append(rvq)
    np.testing.assert_array_equal(out_dev.cpu().numpy(), np.stack(want))
    np.testing.assert_array_equal(ctx_dev.cpu().numpy(), ctx)


# ---------------------------------------------------------------------------
# wide bf16 streams (> 8 rows): RMSNorm + tcgen05 GEMM projections
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("ksplit", ["1", "8"])
def test_wide_stream_step_api_matches_oracle(mrtdf, oracle, tiny_weights, ksplit):
    """ksplit 8: the tcgen05 decode GEMMs may split K over a thread-block
    cluster (the tiny FFN-down takes a 2-way split)."""
    old = os.environ.get("MRTDF_WIDE_KSPLIT")
    os.environ["MRTDF_WIDE_KSPLIT"] = ksplit
    try:
        cfg, eng = _engine(mrtdf, tiny_weights, "tiny", 1)
    finally:
        if old is None:
            del os.environ["MRTDF_WIDE_KSPLIT"]
        else:
            os.environ["MRTDF_WIDE_KSPLIT"] = old
    nseq = 8  # 16 rows
    ids = np.concatenate([random_ids(cfg, 2, 60, seed=50 + i) for i in range(nseq)])
    st = mrtdf.Stream(eng, nseq, True)
    assert st.rows == 16
    orc = oracle.Oracle(tiny_weights, cfg.as_ints())
    st.encode(ids)
    orc.encode(ids)
    rng = np.random.default_rng(5)
    x = None
    for f in range(3):
        a = st.temporal_step(x, f)
        b = orc.temporal_step(x, f)
        assert np.abs(a - b).max() <= BF16_TOL * 4, f
        d = None
        for l in range(4):
            la = st.depth_step(d, l)
            lb = orc.depth_step(d, l)
            assert np.abs(la - lb).max() <= BF16_TOL, (f, l)
            d = rng.standard_normal((16, cfg.d_model)).astype(np.float32) * 0.5
        x = rng.standard_normal((16, cfg.d_model)).astype(np.float32) * 0.5


def test_wide_stream_generation(mrtdf, tiny_weights):
    """64 CFG pairs in one stream: tokens in their level ranges, graph replay
    equal to stream launches, sequence i independent of its neighbours."""
    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", 1)
    nseq = 64
    ids = np.concatenate([random_ids(cfg, 2, cfg.max_encoder_length, seed=60 + i % 4) for i in range(nseq)])
    st = mrtdf.Stream(eng, nseq, True)
    o = mrtdf.gen_opts(cfg, cfg.max_frames, seed=7)
    seeds = [100 + (i % 4) for i in range(nseq)]
    a = st.generate_tokens(ids, o, seeds=seeds)
    b = st.generate_tokens(ids, o, seeds=seeds)  # graph replay
    np.testing.assert_array_equal(a, b)
    lo = cfg.codec_offset + np.arange(cfg.rvq_depth) * cfg.codebook_size
    assert ((a >= lo) & (a < lo + cfg.codebook_size)).all()
    # sequences with the same ids and seed decode the same tokens
    for i in range(4, nseq):
        np.testing.assert_array_equal(a[i], a[i % 4])


def test_wide_stream_hybrid_matches_narrow(mrtdf):
    """Full-size wide stream (split-K cluster GEMMs: 96 / 88 / 64 CTAs per
    projection) against the 2-row GEMV path on the same rows. Both are bf16
    with different fp32 accumulation orders, so the bound is the bf16 noise
    floor: each is compared with the fp32 engine and the wide path may not be
    further from it than 1.25 x the 2-row path (mean and max)."""
    ids2 = random_ids(mrtdf.preset("hybrid", 1), 2, 256, seed=70)
    outs = {}
    for name, dtype, nseq in (("wide", 1, 8), ("narrow", 1, 1), ("fp32", 0, 1)):
        cfg = mrtdf.preset("hybrid", dtype)
        eng = mrtdf.Engine(cfg).load_random(0)
        st = mrtdf.Stream(eng, nseq, True)
        st.encode(np.concatenate([ids2] * nseq))
        t = st.temporal_step(None, 0)
        lg = st.depth_step(None, 0)
        outs[name] = (t, lg)
        st.close()
        eng.close()
    tw, lw = outs["wide"]
    np.testing.assert_array_equal(tw[:2], tw[14:])  # identical rows stay identical
    for k in range(2):
        w, n, f = outs["wide"][k][:2], outs["narrow"][k], outs["fp32"][k]
        ew, en = np.abs(w - f), np.abs(n - f)
        msg = (k, ew.mean(), en.mean(), ew.max(), en.max(), np.abs(w - n).max())
        assert ew.mean() <= 1.25 * en.mean() + 1e-3, msg
        assert ew.max() <= 1.25 * en.max() + 2e-2, msg


def test_chunk_graph_kernel_count(mrtdf, tiny_weights):
    """The chunk graph holds exactly the kernels the structure implies (the
    bench's gpu_launches claim): encoder, PAD embedding, then per frame the
    temporal layers and 16 x (depth layers + lm_head + sampler)."""
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench

    cfg, eng = _engine(mrtdf, tiny_weights, "tiny", 1)
    st = mrtdf.Stream(eng, 1, True)
    ids = random_ids(cfg, 2, cfg.max_encoder_length, seed=80)
    st.generate_tokens(ids, mrtdf.gen_opts(cfg, cfg.max_frames, seed=1))
    assert st.chunk_kernels() == bench.st_launch_count(cfg, cfg.max_frames, fused=True)

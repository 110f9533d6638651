"""mrtdf_sample_noalloc: the sampler on caller-owned device buffers, with its
scratch in a fixed device array of the library instead of cudaMalloc'd
temporaries. Its tokens must equal mrtdf_sample's on the same logits, draws
and options, for two calls queued back to back before one synchronise.

The file name sorts last so that the test also runs after every other GPU
test in the same process (the array is set up once per device)."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

SCRATCH_ROW_BYTES = 21760  # per feedback row; rows x d_model x dtype bytes above it is rejected


def _cases(cfg, rng, n):
    V = cfg.vocab_size
    for trial in range(n):
        rows = 1 + trial % 2
        logits = rng.standard_normal((rows, V)).astype(np.float32) * 3
        if trial % 3 == 0:
            logits = np.round(logits * 2) / 2  # ties at the top-k threshold
        T = [0.0, 1.1, 0.5, 2.0][trial % 4]
        k = [40, 1, 0, 64, 7][trial % 5]
        masked = trial % 7 != 0
        level = trial % cfg.rvq_depth
        frame = trial % 5
        u = rng.uniform(1e-7, 1 - 1e-7, V).astype(np.float32) if trial % 2 == 0 else None
        yield logits, T, k, masked, level, frame, 1000 + trial, u


def _check_pairs(mrtdf, cfg, eng, rng, n):
    cases = list(_cases(cfg, rng, n))
    for i in range(0, len(cases) - 1, 2):
        pair = cases[i:i + 2]
        opts = [mrtdf.gen_opts(cfg, 1, temperature=T, top_k=k, guidance_weight=4.0, use_vocab_masks=masked, seed=seed)
                for (_, T, k, masked, _, _, seed, _) in pair]
        want = [eng.sample(c[0], c[5], c[4], o, uniforms=c[7]) for c, o in zip(pair, opts)]
        dev = [(torch.from_numpy(c[0]).to("cuda:0"), None if c[7] is None else torch.from_numpy(c[7]).to("cuda:0"))
               for c in pair]
        tok = torch.full((2,), -1, dtype=torch.int32, device="cuda:0")
        torch.cuda.synchronize()
        # two calls in a row on the legacy default stream, one synchronise after both
        for j, ((logits, _, _, _, level, frame, _, _), o, (dl, du)) in enumerate(zip(pair, opts, dev)):
            eng.sample_noalloc(dl.data_ptr(), logits.shape[0] == 2, frame, level, o,
                               None if du is None else du.data_ptr(), tok[j:].data_ptr(), 0)
        torch.cuda.synchronize()
        got = tok.cpu().tolist()
        assert got == want, (i, got, want)


@pytest.mark.parametrize("dtype", [0, 1])
def test_noalloc_sample_equals_sample_tiny(mrtdf, tiny_weights, dtype):
    cfg = mrtdf.preset("tiny", dtype)
    eng = mrtdf.Engine(cfg).load_safetensors(tiny_weights)
    _check_pairs(mrtdf, cfg, eng, np.random.default_rng(40 + dtype), 60)


def test_noalloc_sample_equals_sample_hybrid(mrtdf):
    cfg = mrtdf.preset("hybrid", mrtdf.DTYPE_BF16)
    eng = mrtdf.Engine(cfg).load_random(0)
    _check_pairs(mrtdf, cfg, eng, np.random.default_rng(50), 12)


def test_noalloc_reports_a_failed_draw(mrtdf, tiny_weights):
    """The call returns before the draw, so a draw without a valid candidate
    (NaN logits) is reported in the result: the token is -1. A good draw
    right after it on the same stream is unaffected."""
    cfg = mrtdf.preset("tiny", mrtdf.DTYPE_BF16)
    eng = mrtdf.Engine(cfg).load_safetensors(tiny_weights)
    bad = torch.full((2, cfg.vocab_size), float("nan"), dtype=torch.float32, device="cuda:0")
    good_h = np.random.default_rng(3).standard_normal((2, cfg.vocab_size)).astype(np.float32)
    good = torch.from_numpy(good_h).to("cuda:0")
    tok = torch.full((2,), 7, dtype=torch.int32, device="cuda:0")
    o = mrtdf.gen_opts(cfg, 1, temperature=1.1, top_k=40, guidance_weight=4.0, seed=5)
    torch.cuda.synchronize()
    eng.sample_noalloc(bad.data_ptr(), True, 0, 2, o, None, tok[0:].data_ptr(), 0)
    eng.sample_noalloc(good.data_ptr(), True, 0, 2, o, None, tok[1:].data_ptr(), 0)
    torch.cuda.synchronize()
    got = tok.cpu().tolist()
    assert got[0] == -1
    assert got[1] == eng.sample(good_h, 0, 2, o)


def test_noalloc_rejects_rows_beyond_scratch(mrtdf):
    # fp32, CFG pair: 2 x 2752 x 4 bytes = 22016 > the fixed 21760-byte row
    cfg = mrtdf.preset("tiny", mrtdf.DTYPE_FP32, d_model=2752)
    eng = mrtdf.Engine(cfg).load_random(0)
    dl = torch.zeros((2, cfg.vocab_size), dtype=torch.float32, device="cuda:0")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    o = mrtdf.gen_opts(cfg, 1)
    with pytest.raises(mrtdf.MrtdfError) as e:
        eng.sample_noalloc(dl.data_ptr(), True, 0, 0, o, None, tok.data_ptr(), 0)
    assert e.value.code == 7 and "fixed scratch" in str(e.value)
    # a single row (1 x 2752 x 4 = 11008 bytes) fits
    eng.sample_noalloc(dl.data_ptr(), False, 0, 0, o, None, tok.data_ptr(), 0)
    torch.cuda.synchronize()
    assert 2 <= int(tok.item()) < 2 + cfg.codebook_size

"""CPU checks of the SpectroStream decode-phase oracle (oracle/
spectrostream_oracle.cpp) against an independent torch / numpy formulation
of the same reference code: conv2d and conv_transpose2d layers, the causal
padding arithmetic, the iSTFT (also as a round trip through a restated
stft_preprocess), RVQ dequantisation, and the whole decoder at a small
number of frames. No GPU needed."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
F = torch.nn.functional

# Decoder block table, spectrostream.cpp:328-338: in, out, stride, transposed kernel
DEC = [(512, 1024, (2, 1), (4, 3)), (512, 256, (2, 2), (4, 4)), (256, 256, (1, 2), (3, 4)),
       (256, 256, (1, 2), (3, 4)), (256, 128, (1, 3), (3, 6)), (128, 128, (1, 2), (3, 4)),
       (128, 64, (1, 2), (3, 4))]


@pytest.fixture(scope="module")
def codec_bundle(mrtdf, tmp_path_factory):
    import mrtss

    d = tmp_path_factory.mktemp("codec")
    dec, cb = str(d / "spectrostream_decoder.safetensors"), str(d / "codebooks.safetensors")
    mrtss.write_random_safetensors(7, 16, dec, cb)
    return dec, cb


def _nchw(x):
    return torch.from_numpy(np.ascontiguousarray(x)).permute(0, 3, 1, 2)


def _nhwc(t):
    return t.permute(0, 2, 3, 1).contiguous().numpy()


def _causal_pad_t(x, kh, kw, sh, sw):
    # causal_same_pad (spectrostream.cpp:41-62) on an NCHW tensor
    W = x.shape[3]
    ow = -(-W // sw)
    tot = max((ow - 1) * sw + kw - W, 0)
    return F.pad(x, (tot // 2, tot - tot // 2, kh - sh, 0))


def _close(a, b, rel=2e-5):
    scale = max(float(np.abs(b).max()), 1e-6)
    err = float(np.abs(a - b).max()) / scale
    assert err < rel, (err, scale)


@pytest.mark.parametrize("k,s", [((3, 3), (1, 1)), ((7, 7), (1, 1)), ((3, 4), (1, 2)), ((4, 4), (2, 2)),
                                 ((1, 1), (1, 1))])
def test_conv2d_matches_torch(oracle, k, s):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 9, 13, 40)).astype(np.float32)
    w = rng.standard_normal((24, 40, *k)).astype(np.float32) * 0.1
    b = rng.standard_normal(24).astype(np.float32)
    for causal in (False, True):
        got = oracle.conv2d(x, w, b, s, causal_pad=causal)
        xt = _nchw(x)
        if causal:
            xt = _causal_pad_t(xt, k[0], k[1], s[0], s[1])
        want = _nhwc(F.conv2d(xt, torch.from_numpy(w), torch.from_numpy(b), stride=s))
        assert got.shape == want.shape
        _close(got, want)


def test_causal_same_pad_shapes(oracle):
    # output width = ceil(W / sw), height = H / sh (H padded on top by kh - sh)
    rng = np.random.default_rng(2)
    x = rng.standard_normal((1, 8, 11, 8)).astype(np.float32)
    for (kh, kw), (sh, sw) in [((7, 7), (1, 1)), ((3, 4), (1, 2)), ((3, 6), (1, 3)), ((4, 3), (2, 1))]:
        w = np.zeros((8, 8, kh, kw), np.float32)
        y = oracle.conv2d(x, w, np.zeros(8, np.float32), (sh, sw), causal_pad=True)
        assert y.shape[1:3] == ((8 + kh - sh - kh) // sh + 1, -(-11 // sw)), (kh, kw, sh, sw, y.shape)


@pytest.mark.parametrize("k,s", [((4, 3), (2, 1)), ((4, 4), (2, 2)), ((3, 4), (1, 2)), ((3, 6), (1, 3))])
def test_conv_transpose2d_matches_torch(oracle, k, s):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 5, 7, 32)).astype(np.float32)
    w = rng.standard_normal((32, 16, *k)).astype(np.float32) * 0.1  # (I, O, kh, kw)
    b = rng.standard_normal(16).astype(np.float32)
    got = oracle.conv_transpose2d(x, w, b, s)
    want = _nhwc(F.conv_transpose2d(_nchw(x), torch.from_numpy(w), torch.from_numpy(b), stride=s))
    assert got.shape == want.shape
    _close(got, want)


def _hann_synth():
    # istft_postprocess window arithmetic (spectrostream.cpp:627-637), float32
    t = np.arange(960, dtype=np.float32)
    win = (np.float32(0.5) - np.float32(0.5) * np.cos(t * np.float32(2 * np.pi / 960))).astype(np.float32)
    per = (win * win).reshape(2, 480).sum(0)
    return win, win / np.concatenate([per, per])


def test_istft_matches_numpy(oracle):
    rng = np.random.default_rng(4)
    B, H = 2, 6
    spec = rng.standard_normal((B, H, 480, 4)).astype(np.float32)
    target = H * 480 + 200
    got = oracle.istft(spec, target)
    _, synth = _hann_synth()
    want = np.zeros((B, target, 2), np.float64)
    for b in range(B):
        for s in range(2):
            X = spec[b, :, :, 2 * s].astype(np.float64) + 1j * spec[b, :, :, 2 * s + 1]
            X = np.concatenate([X, np.zeros((H, 1))], axis=1)  # Nyquist bin
            fr = np.fft.irfft(X, n=960, axis=-1) * synth
            audio = np.zeros((H + 1) * 480)
            for i in range(H):
                audio[i * 480:i * 480 + 960] += fr[i]
            want[b, :, s] = audio[:target]
    _close(got, want.astype(np.float32), rel=2e-6)


def test_istft_inverts_stft_preprocess(oracle):
    # stft_preprocess (spectrostream.cpp:511-591) restated in numpy, then the
    # oracle's iSTFT: band-limited stereo audio comes back in the interior
    # (the first hop has no overlap partner; the Nyquist bin is dropped).
    T = 480 * 12 + 960
    n = np.arange(T)
    audio = np.stack([np.sin(2 * np.pi * 440 * n / 48000) + 0.3 * np.cos(2 * np.pi * 3000 * n / 48000),
                      0.5 * np.sin(2 * np.pi * 1234.5 * n / 48000)], axis=-1).astype(np.float32)
    win, _ = _hann_synth()
    frames = (T - 960) // 480 + 1
    spec = np.zeros((1, frames, 480, 4), np.float32)
    for s in range(2):
        fr = np.stack([audio[i * 480:i * 480 + 960, s] * win for i in range(frames)])
        X = np.fft.rfft(fr, n=960, axis=-1)[:, :480]
        spec[0, :, :, 2 * s] = X.real
        spec[0, :, :, 2 * s + 1] = X.imag
    rec = oracle.istft(spec, frames * 480 + 480)[0]
    assert np.abs(rec[480:frames * 480] - audio[480:frames * 480]).max() < 1e-4


def test_dequantize_matches_numpy(oracle, codec_bundle):
    from safetensors.numpy import load_file

    cb = load_file(codec_bundle[1])["codebooks"]
    assert cb.shape == (16, 1024, 256)
    rng = np.random.default_rng(5)
    codes = rng.integers(0, 1024, size=(7, 16), dtype=np.int32)
    o = oracle.CodecOracle(*codec_bundle)
    got = o.rvq_dequantize(codes)
    want = np.zeros((7, 256), np.float32)
    for k in range(16):  # rvq.cpp:80-84, float32 adds in level order
        want = want + cb[k][codes[:, k]]
    np.testing.assert_array_equal(got, want)
    with pytest.raises(RuntimeError):
        o.rvq_dequantize(np.full((1, 16), 1024, np.int32))


def _torch_decoder(w, emb):
    """SpectroStreamDecoder::operator() (spectrostream.cpp:365-419) written
    with torch NCHW ops from the canonical weights."""
    def conv(x, p, pad=None, stride=(1, 1)):
        if pad is not None:
            x = _causal_pad_t(x, *pad, 1, 1)
        return F.conv2d(x, torch.from_numpy(w[p + ".weight"]), torch.from_numpy(w[p + ".bias"]), stride=stride)

    elu = F.elu
    B, S, _ = emb.shape
    x = torch.from_numpy(emb)
    x = torch.cat([x, torch.zeros(B, 1, 256)], dim=1)          # (B, S+1, 256)
    x = x[:, :, None, :].permute(0, 3, 1, 2)                    # NCHW (B, 256, S+1, 1)
    skip = conv(x, "input_proj.shortcut")
    m = conv(elu(conv(x, "input_proj.conv1")), "input_proj.conv2")
    x = m + skip                                                # (B, 2560, S+1, 1)
    # unfold_width(5): NHWC reshape (B, H, 1, 2560) -> (B, H, 5, 512)
    xh = x.permute(0, 2, 3, 1).reshape(B, S + 1, 5, 512)
    x = xh.permute(0, 3, 1, 2)
    y = conv(elu(conv(elu(x), "input_conv.conv1", (3, 3))), "input_conv.conv2", (3, 3))
    x = y + x
    for i, (cin, cout, (sh, sw), (kh, kw)) in enumerate(DEC):
        p = f"decoder_blocks.{i}"
        y = F.conv_transpose2d(elu(x), torch.from_numpy(w[p + ".conv_transpose.weight"]),
                               torch.from_numpy(w[p + ".conv_transpose.bias"]), stride=(sh, sw))
        ch, cw = kh - sh, kw - sw
        y = y[:, :, :y.shape[2] - ch, cw // 2:y.shape[3] - (cw - cw // 2)]
        y = conv(elu(y), p + ".conv", (3, 3))
        r = x.repeat_interleave(sh, dim=2).repeat_interleave(sw, dim=3)
        if cin != cout:
            r = conv(r, p + ".shortcut")
        x = y + r
        if i == 0:  # stereo split: channel block s -> image s * B + b
            Bx, C, H, W = x.shape
            x = x.reshape(Bx, 2, C // 2, H, W).permute(1, 0, 2, 3, 4).reshape(2 * Bx, C // 2, H, W)
    x = conv(elu(x), "output_conv", (7, 7))[:, :, 4:]          # (2B, 2, H, 480)
    x = x.permute(0, 2, 3, 1)                                   # (2B, H, 480, 2)
    H, W = x.shape[1:3]
    x = x.reshape(2, B, H, W, 2).permute(1, 2, 3, 0, 4).reshape(B, H, W, 4)
    return x.numpy()


def test_decoder_matches_torch_formulation(oracle, codec_bundle):
    from safetensors.numpy import load_file

    w = load_file(codec_bundle[0])
    rng = np.random.default_rng(6)
    emb = rng.standard_normal((1, 2, 256)).astype(np.float32)
    o = oracle.CodecOracle(*codec_bundle)
    got = o.decode(emb)
    assert got.shape == (1, 8, 480, 4)
    with torch.no_grad():
        want = _torch_decoder(w, emb)
    assert want.shape == got.shape
    assert np.isfinite(got).all() and np.abs(got).max() > 1e-3
    _close(got, want, rel=1e-4)


def test_decode_tokens_is_the_composition(oracle, codec_bundle):
    rng = np.random.default_rng(8)
    codes = rng.integers(0, 1024, size=(2, 16), dtype=np.int32)
    o = oracle.CodecOracle(*codec_bundle)
    audio = o.decode_tokens(codes)
    assert audio.shape == (2 * 1920, 2)
    spec = o.decode(o.rvq_dequantize(codes)[None])
    np.testing.assert_array_equal(audio, oracle.istft(spec, 2 * 1920)[0])


def test_random_codec_bundle_layout(codec_bundle):
    """Keys and canonical shapes the reference's constructors read
    (spectrostream.cpp:125-157, 163-222, 356-363; system.cpp:372-373)."""
    from safetensors.numpy import load_file

    w = load_file(codec_bundle[0])
    assert w["input_proj.conv1.weight"].shape == (2560, 256, 1, 1)
    assert w["input_proj.conv2.weight"].shape == (2560, 2560, 1, 1)
    assert w["input_proj.shortcut.weight"].shape == (2560, 256, 1, 1)
    assert w["input_conv.conv2.weight"].shape == (512, 512, 3, 3)
    for i, (cin, cout, _, (kh, kw)) in enumerate(DEC):
        p = f"decoder_blocks.{i}"
        assert w[p + ".conv_transpose.weight"].shape == (cin, cout, kh, kw)  # (I, O, kh, kw)
        assert w[p + ".conv.weight"].shape == (cout, cout, 3, 3)
        assert (p + ".shortcut.weight" in w) == (cin != cout)
        assert w[p + ".conv.bias"].shape == (cout,)
    assert w["output_conv.weight"].shape == (2, 64, 7, 7)
    assert all(v.dtype == np.float32 for v in w.values())
    # fan-in scaled init keeps the residual stack's activations O(1)
    s = w["decoder_blocks.1.conv.weight"].std()
    assert abs(s - 1 / np.sqrt(256 * 9)) < 0.1 / np.sqrt(256 * 9)

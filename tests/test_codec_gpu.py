"""GPU parity of the SpectroStream decode phase (include/mrtss.h) against the
CPU oracle (oracle/spectrostream_oracle.cpp), through the C ABI.

Tolerances: the decoder's convolutions run on the tensor cores with tf32
operands (10-bit mantissa) and float32 accumulation, against a float32
oracle, so the decoder output and the audio are compared by relative L2
error (< 2e-2) and max error relative to the largest value (< 5e-2); the
iSTFT (float32 SIMT) to 1e-4 of the largest value; RVQ dequantisation
(float32 adds in the reference's order) bit-exactly."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mrtss_mod(mrtdf):
    import mrtss

    return mrtss


@pytest.fixture(scope="module")
def codec_bundle(mrtss_mod, tmp_path_factory):
    d = tmp_path_factory.mktemp("codec_gpu")
    dec, cb = str(d / "spectrostream_decoder.safetensors"), str(d / "codebooks.safetensors")
    mrtss_mod.write_random_safetensors(11, 16, dec, cb)
    return dec, cb


@pytest.fixture(scope="module")
def codec(mrtss_mod, codec_bundle):
    return mrtss_mod.Codec(max_batch=2, max_frames=51).load_safetensors(*codec_bundle)


@pytest.fixture(scope="module")
def codec_oracle(oracle, codec_bundle):
    return oracle.CodecOracle(*codec_bundle)


def _rel(got, want):
    l2 = float(np.linalg.norm((got - want).ravel()) / max(np.linalg.norm(want.ravel()), 1e-12))
    mx = float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-12))
    return l2, mx


def test_dequantize_bit_exact(codec, codec_oracle):
    rng = np.random.default_rng(20)
    codes = rng.integers(0, 1024, size=(37, 16), dtype=np.int32)
    np.testing.assert_array_equal(codec.rvq_dequantize(codes), codec_oracle.rvq_dequantize(codes))
    np.testing.assert_array_equal(codec.rvq_dequantize(codes[:, :5]), codec_oracle.rvq_dequantize(codes[:, :5]))


@pytest.mark.parametrize("B,S", [(1, 1), (1, 3), (2, 2)])
def test_decoder_matches_oracle(codec, codec_oracle, B, S):
    rng = np.random.default_rng(30 + S)
    emb = rng.standard_normal((B, S, 256)).astype(np.float32)
    got = codec.decode(emb)
    want = codec_oracle.decode(emb)
    assert got.shape == want.shape == (B, 4 * S, 480, 4)
    assert np.isfinite(got).all()
    l2, mx = _rel(got, want)
    print(f"decoder B={B} S={S}: rel L2 {l2:.2e}, max {mx:.2e}")
    assert l2 < 2e-2 and mx < 5e-2, (l2, mx)


def test_istft_matches_oracle(codec, oracle):
    rng = np.random.default_rng(40)
    spec = rng.standard_normal((2, 12, 480, 4)).astype(np.float32)
    for target in (12 * 480, 12 * 480 + 300, 1000):
        got = codec.istft(spec, target)
        want = oracle.istft(spec, target)
        err = np.abs(got - want).max() / np.abs(want).max()
        print(f"istft target {target}: max rel {err:.2e}")
        assert err < 1e-4


def test_decode_tokens_full_chunk_matches_oracle(codec, codec_oracle):
    # one production chunk: 50 frames + 1 crossfade frame, 16 levels (system.cpp:289-313)
    rng = np.random.default_rng(50)
    codes = rng.integers(0, 1024, size=(51, 16), dtype=np.int32)
    got = codec.decode_tokens(codes)
    want = codec_oracle.decode_tokens(codes)
    assert got.shape == want.shape == (51 * 1920, 2)
    l2, mx = _rel(got, want)
    print(f"full chunk audio: rel L2 {l2:.2e}, max {mx:.2e}")
    assert l2 < 2e-2 and mx < 5e-2, (l2, mx)


def test_batched_and_device_calls_equal_single(codec):
    rng = np.random.default_rng(60)
    codes = rng.integers(0, 1024, size=(2, 5, 16), dtype=np.int32)
    both = codec.decode_tokens(codes)
    for b in range(2):
        np.testing.assert_array_equal(both[b], codec.decode_tokens(codes[b]))
    dcodes = torch.from_numpy(codes).to("cuda:0")
    daudio = torch.empty((2, 5 * 1920, 2), dtype=torch.float32, device="cuda:0")
    torch.cuda.synchronize()
    codec.decode_tokens_dev(dcodes.data_ptr(), 2, 5, 16, daudio.data_ptr())
    codec.sync()
    np.testing.assert_array_equal(daudio.cpu().numpy(), both)


def test_codec_errors(mrtss_mod, mrtdf, codec):
    with pytest.raises(mrtdf.MrtdfError) as e:
        codec.decode_tokens(np.full((3, 16), 1024, np.int32))
    assert e.value.code == 7
    with pytest.raises(mrtdf.MrtdfError) as e:
        codec.decode_tokens(np.zeros((52, 16), np.int32))  # beyond max_frames
    assert e.value.code == 7
    with pytest.raises(mrtdf.MrtdfError) as e:
        codec.decode_tokens(np.zeros((3, 17), np.int32))  # more levels than codebooks
    assert e.value.code == 1
    c2 = mrtss_mod.Codec(max_batch=1, max_frames=4)
    with pytest.raises(mrtdf.MrtdfError) as e:
        c2.decode_tokens(np.zeros((2, 16), np.int32))
    assert e.value.code == 4  # weights not loaded
    # kernels of one decode: dequant, input_proj 3, input_conv 2, blocks
    # 4 + 6 + 3 + 3 + 5 + 3 + 4 (shortcut, transposed-conv phases, post conv),
    # output conv, iSTFT frames + overlap-add
    assert codec.decode_kernels(1, 51) == 1 + 3 + 2 + 28 + 1 + 2

"""Regenerate tests/golden/codec_golden.npz from the SpectroStream oracle.

    python tests/golden/make_codec_golden.py

The reference ships no SpectroStream test vectors and cannot run here (MLX),
so these fixtures are outputs of the float32 oracle (oracle/
spectrostream_oracle.cpp) on the seed-7 random-init decoder and codebook
bundles (16 levels): RVQ dequantisation, the decoder at 2 codec frames, the
whole codec block on the same codes, and the iSTFT of a fixed spectrogram.
They pin the oracle against regressions (tests/test_golden.py). The sha256
of both bundles is stored so a change of the weight generator is caught.
"""
from __future__ import annotations

import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "magenta-realtime-mlx-cpp_b200"), os.path.join(ROOT, "oracle")]

OUT = os.path.join(HERE, "codec_golden.npz")
SEED, LEVELS, FRAMES = 7, 16, 2


def inputs():
    rng = np.random.default_rng(70)
    codes = rng.integers(0, 1024, size=(FRAMES, LEVELS), dtype=np.int32)
    spec = rng.standard_normal((1, 6, 480, 4)).astype(np.float32)
    return codes, spec


def make(dec_path: str, cb_path: str) -> dict:
    import oracle_py

    codes, spec = inputs()
    o = oracle_py.CodecOracle(dec_path, cb_path)
    emb = o.rvq_dequantize(codes)
    return {
        "codes": codes,
        "spec_in": spec,
        "dequant": emb,
        "decoded": o.decode(emb[None]),
        "audio": o.decode_tokens(codes),
        "istft": oracle_py.istft(spec, 6 * 480 + 100),
    }


def bundles(td: str):
    import mrtss

    dec, cb = os.path.join(td, "d.safetensors"), os.path.join(td, "c.safetensors")
    mrtss.write_random_safetensors(SEED, LEVELS, dec, cb)
    return dec, cb


def main():
    with tempfile.TemporaryDirectory() as td:
        dec, cb = bundles(td)
        shas = [hashlib.sha256(open(p, "rb").read()).hexdigest() for p in (dec, cb)]
        data = make(dec, cb)
    np.savez_compressed(OUT, decoder_sha256=np.array(shas[0]), codebooks_sha256=np.array(shas[1]), **data)
    print(OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()

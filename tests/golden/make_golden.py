"""Regenerate tests/golden/tiny_golden.npz from the CPU oracle.

    python tests/golden/make_golden.py

The reference itself (MLX) cannot run here and ships no golden vectors for
the Depthformer path, so these fixtures are oracle outputs on the tiny
config with the seed-0 random-init bundle. They pin the oracle against
regressions (tests/test_golden.py, CPU) and give the GPU tests a fixed
target. The sha256 of the weight bundle is stored so a change of the
generator is caught instead of silently changing every fixture.
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

OUT = os.path.join(HERE, "tiny_golden.npz")


def inputs(cfg):
    rng = np.random.default_rng(1)
    ids = rng.integers(0, cfg.vocab_size, size=(1, cfg.max_encoder_length)).astype(np.int32)
    ids = np.repeat(ids, 2, 0)
    ids[1, -6:] = 1
    rng = np.random.default_rng(2)
    forced = np.stack([cfg.codec_offset + np.arange(cfg.rvq_depth) * cfg.codebook_size
                       + rng.integers(0, cfg.codebook_size, cfg.rvq_depth) for _ in range(2)]).astype(np.int32)
    return ids, forced


def make(path_weights: str, cfg32, cfg16):
    import oracle_py

    ids, forced = inputs(cfg32)
    o32 = oracle_py.Oracle(path_weights, cfg32.as_ints())
    o16 = oracle_py.Oracle(path_weights, cfg16.as_ints())
    F = cfg32.max_frames
    return {
        "ids": ids,
        "forced": forced,
        "tf_logits_fp32": o32.teacher_forced(ids, forced, 1),
        "tf_logits_bf16": o16.teacher_forced(ids, forced, 1),
        "greedy_fp32": o32.generate(ids, F, 4.0, 0.0, 40, True, 0),
        "greedy_fp32_nocfg": o32.generate(ids[:1], F, 4.0, 0.0, 40, True, 0),
        "sampled_fp32_seed1": o32.generate(ids, F, 4.0, 1.1, 40, True, 1),
        "sampled_bf16_seed1": o16.generate(ids, F, 4.0, 1.1, 40, True, 1),
    }


def main():
    import mrtdf

    cfg32 = mrtdf.preset("tiny", mrtdf.DTYPE_FP32)
    cfg16 = mrtdf.preset("tiny", mrtdf.DTYPE_BF16)
    with tempfile.TemporaryDirectory() as td:
        wpath = os.path.join(td, "tiny.safetensors")
        mrtdf.write_random_safetensors(cfg32, 0, wpath)
        sha = hashlib.sha256(open(wpath, "rb").read()).hexdigest()
        data = make(wpath, cfg32, cfg16)
    np.savez_compressed(OUT, weights_sha256=np.array(sha), **data)
    print(OUT, os.path.getsize(OUT), "bytes; weights sha256", sha)


if __name__ == "__main__":
    main()

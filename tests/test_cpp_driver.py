"""The C++ side of the boundary: include/mrtdf.hpp (the reference's
Depthformer argument order and exception types over the C ABI) and the C++
dry-run driver built on it (the reference CLI's chunk loop,
cli/main.cpp:436-516). CPU: the header compiles on its own. GPU: the driver's
tokens equal the same System loop driven through mrtdf_generate_tokens."""
from __future__ import annotations

import json
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DRIVER = os.path.join(ROOT, "magenta-realtime-mlx-cpp_b200", "lib", "mrtdf_dry_run")


def test_cpp_header_compiles_alone(tmp_path):
    src = tmp_path / "use.cpp"
    src.write_text('#include "mrtdf.hpp"\n'
                   'int main() { mrtdf::GenerateOptions o; mrtdf::IntArray a({2, 3});\n'
                   '  return (o.num_frames == 50 && a.numel() == 6) ? 0 : 1; }\n')
    r = subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-fsyntax-only", "-I", os.path.join(ROOT, "include"),
                        str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_driver_is_built(mrtdf):
    assert os.access(DRIVER, os.X_OK)


def _splitmix_style(seed: int, n: int, cfg) -> np.ndarray:
    mask = (1 << 64) - 1
    x = seed
    out = []
    for _ in range(n):
        x = (x + 0x9E3779B97F4A7C15) & mask
        z = x
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & mask
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & mask
        z ^= z >> 31
        out.append(cfg.codec_offset + z % (cfg.rvq_depth * cfg.codebook_size))
    return np.array(out, np.int32)


@pytest.mark.gpu
def test_cpp_dry_run_matches_generate_tokens(mrtdf, tiny_weights, tmp_path):
    out = tmp_path / "ids.bin"
    W, N, seed, style_seed = 2, 3, 5, 9
    r = subprocess.run([DRIVER, "--preset", "tiny", "--weights", tiny_weights, "--chunks", str(N), "--warmup", str(W),
                        "--seed", str(seed), "--style-seed", str(style_seed), "--out", str(out)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    assert f"dry-run: {N} chunks" in r.stderr and "p99=" in r.stderr, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["chunks"] == N and line["rtf"] > 0
    cfg = mrtdf.preset("tiny", mrtdf.DTYPE_BF16)
    F = min(cfg.max_frames, (cfg.max_encoder_length - 6) // 4)
    got = np.fromfile(out, np.int32).reshape(N, F, cfg.rvq_depth)
    # the same System loop through the C ABI (Python mirror)
    eng = mrtdf.Engine(cfg).load_safetensors(tiny_weights)
    st = mrtdf.Stream(eng, 1, True)
    ctx = -np.ones(((cfg.max_encoder_length - 6) // 4, cfg.rvq_depth), np.int32)
    style = _splitmix_style(style_seed, 6, cfg)
    want = []
    for chunk in range(W + N):
        enc = mrtdf.build_encoder_inputs(ctx, style, 4, cfg.codebook_size, cfg.codec_offset)
        toks = st.generate_tokens(enc, mrtdf.gen_opts(cfg, F, temperature=1.1, top_k=40, guidance_weight=4.0,
                                                      seed=seed + chunk))[0]
        ctx = mrtdf.context_roll(ctx, mrtdf.llm_to_rvq(toks, cfg.codebook_size, cfg.codec_offset))
        if chunk >= W:
            want.append(toks)
    np.testing.assert_array_equal(got, np.stack(want))


@pytest.mark.gpu
def test_cpp_driver_reports_errors(mrtdf, tmp_path):
    """A missing weight bundle fails with the library's message, as a
    std::runtime_error (exit 2); a bundle without the needed keys is a
    missing key, std::out_of_range (exit 3), as weights.cpp:40-41 throws."""
    r = subprocess.run([DRIVER, "--preset", "tiny", "--weights", str(tmp_path / "none.safetensors")],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 2 and "none.safetensors" in r.stderr, r.stderr
    small = tmp_path / "small.safetensors"
    mrtdf.write_random_safetensors(mrtdf.preset("tiny", 1, num_depth_layers=1), 0, str(small))
    r = subprocess.run([DRIVER, "--preset", "tiny", "--weights", str(small)], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 3 and "missing key" in r.stderr, r.stderr

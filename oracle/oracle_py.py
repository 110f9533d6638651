"""ctypes bindings of the CPU oracle (oracle/_build/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by bench.py's CPU-baseline
legs and by __graft_entry__.smoke() as the checker. The engine never uses it.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        from build_oracle import build  # noqa: E402  (same directory)

        path = build()
        L = ctypes.CDLL(path)
        L.orc_last_error.restype = ctypes.c_char_p
        L.orc_create.restype = ctypes.c_void_p
        L.orc_create.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_int)]
        L.orc_destroy.argtypes = [ctypes.c_void_p]
        for n in ["orc_encode", "orc_temporal_step", "orc_depth_step", "orc_generate", "orc_teacher_forced"]:
            getattr(L, n).restype = ctypes.c_int
        L.orc_encode.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        L.orc_temporal_step.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        L.orc_depth_step.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        L.orc_generate.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                                   ctypes.c_void_p, ctypes.c_void_p]
        L.orc_teacher_forced.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_void_p, ctypes.c_void_p]
        L.orc_sample.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                 ctypes.c_void_p, ctypes.c_void_p]
        L.orc_relative_bucket.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_sinusoid.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        L.orc_bf16_round.restype = ctypes.c_float
        L.orc_bf16_round.argtypes = [ctypes.c_float]
        L.orc_philox_uniform.restype = ctypes.c_float
        L.orc_philox_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32]
        L.orc_philox4x32_10.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.orc_exact_log.restype = ctypes.c_float
        L.orc_exact_log.argtypes = [ctypes.c_float]
        L.orc_gumbel.restype = ctypes.c_float
        L.orc_gumbel.argtypes = [ctypes.c_float]
        L.orc_cfg_mix.restype = ctypes.c_float
        L.orc_cfg_mix.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_float]
        L.orc_gelu.restype = ctypes.c_float
        L.orc_gelu.argtypes = [ctypes.c_float, ctypes.c_int]
        L.orc_set_num_threads.argtypes = [ctypes.c_int]
        L.orc_create_random.restype = ctypes.c_void_p
        L.orc_create_random.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_uint64, ctypes.c_float, ctypes.c_int]
        L.orc_gen_begin.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.orc_gen_frame.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_uint64, ctypes.c_void_p]
        L.orc_embed_pe.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        L.orc_encoder_layer.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_void_p]
        L.orc_decoder_layer.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_void_p]
        L.orc_get_cache.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
        L.orc_set_cache.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_int, ctypes.c_int]
        L.orc_lm_head.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_void_p]
        # SpectroStream decode phase (spectrostream_oracle.cpp)
        P, I = ctypes.c_void_p, ctypes.c_int
        L.orc_ss_last_error.restype = ctypes.c_char_p
        L.orc_ss_create.restype = P
        L.orc_ss_create.argtypes = [ctypes.c_char_p, ctypes.c_char_p]
        L.orc_ss_destroy.argtypes = [P]
        L.orc_ss_dequantize.argtypes = [P, P, I, I, P]
        L.orc_ss_decode.argtypes = [P, P, I, I, P]
        L.orc_ss_istft.argtypes = [P, I, I, I, P]
        L.orc_ss_decode_tokens.argtypes = [P, P, I, I, P]
        L.orc_ss_conv2d.argtypes = [P, I, I, I, I, P, P, I, I, I, I, I, I, P]
        L.orc_ss_conv_transpose2d.argtypes = [P, I, I, I, I, P, P, I, I, I, I, I, P]
        L.orc_ss_set_num_threads.argtypes = [I]
        # MusicCoCa text tower + style RVQ (musiccoca_oracle.cpp)
        L.orc_mc_last_error.restype = ctypes.c_char_p
        L.orc_mc_create.restype = P
        L.orc_mc_create.argtypes = [ctypes.c_char_p, ctypes.c_char_p]
        L.orc_mc_destroy.argtypes = [P]
        L.orc_mc_embed_text.argtypes = [P, P, P, I, I, P]
        L.orc_mc_quantize.argtypes = [P, P, I, I, P]
        _lib = L
    return _lib


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


def _check(rc: int):
    if rc != 0:
        raise RuntimeError("oracle: " + lib().orc_last_error().decode())


# Config field order of include/mrtdf.h (DepthformerConfig, model.h:47-68).
CONFIG_FIELDS = [
    "vocab_size", "d_model", "d_kv", "d_ff", "num_heads", "num_encoder_layers", "num_temporal_layers",
    "num_depth_layers", "max_encoder_length", "rvq_depth", "temporal_num_buckets", "temporal_max_distance",
    "depth_num_buckets", "depth_max_distance", "codebook_size", "codec_offset", "max_frames", "dtype",
]


def preset_ints(name: str, dtype: int = 1) -> list:
    """Model presets as config ints, restated for the CPU arms: "base"
    (DepthformerConfig::base(), model.cpp:34-36), "large" (model.cpp:38-48)
    and "hybrid", the benchmark architecture of BASELINE.json (large widths,
    base depths, 32 / 128 temporal buckets, vocab 16 x 1024 + 4)."""
    c = dict(vocab_size=29824, d_model=768, d_kv=64, d_ff=2048, num_heads=12, num_encoder_layers=12,
             num_temporal_layers=20, num_depth_layers=4, max_encoder_length=1006, rvq_depth=16,
             temporal_num_buckets=128, temporal_max_distance=128, depth_num_buckets=16, depth_max_distance=16,
             codebook_size=1024, codec_offset=2, max_frames=50, dtype=dtype)
    if name == "large":
        c.update(d_model=1024, d_ff=2816, num_heads=16, num_encoder_layers=24, num_temporal_layers=40,
                 num_depth_layers=8)
    elif name == "hybrid":
        c.update(d_model=1024, d_ff=2816, num_heads=16, vocab_size=16388, temporal_num_buckets=32)
    elif name != "base":
        raise ValueError(f"unknown preset {name}")
    return [c[f] for f in CONFIG_FIELDS]


def build_encoder_inputs(context: np.ndarray, style: np.ndarray, enc_depth: int, codebook_size: int,
                         codec_offset: int) -> np.ndarray:
    """build_encoder_inputs_host (system.cpp:62-95): row 0 = the context's
    first enc_depth levels per frame mapped to codec_offset + level *
    codebook_size + code (MASK = 1 where the code is negative), then the
    style ids; row 1 = the same context with the style masked."""
    ctx = np.asarray(context, np.int64)[:, :enc_depth]
    lvl = np.arange(enc_depth, dtype=np.int64)[None, :]
    row = np.where(ctx >= 0, codec_offset + lvl * codebook_size + ctx, 1).reshape(-1)
    style = np.asarray(style, np.int64).reshape(-1)
    out = np.empty((2, row.size + style.size), np.int32)
    out[0] = np.concatenate([row, style])
    out[1] = np.concatenate([row, np.ones_like(style)])
    return out


class Oracle:
    """CPU restatement of the Depthformer (fp32 or bf16-emulating)."""

    def __init__(self, safetensors_path: Optional[str], cfg_ints, _handle=None):
        if _handle is None:
            arr = (ctypes.c_int * 18)(*cfg_ints)
            _handle = lib().orc_create(safetensors_path.encode(), arr)
            if not _handle:
                raise RuntimeError("oracle: " + lib().orc_last_error().decode())
        self.h = _handle
        self.cfg = list(cfg_ints)
        self.V, self.d, self.depth = cfg_ints[0], cfg_ints[1], cfg_ints[9]
        self.rows = 0

    @classmethod
    def from_random(cls, cfg_ints, seed: int, stddev: float = 0.02, norm_ones: bool = True) -> "Oracle":
        """The random-init bundle of `seed` (the oracle's own restatement of
        the generator), built in memory without a file."""
        arr = (ctypes.c_int * 18)(*cfg_ints)
        h = lib().orc_create_random(arr, seed, stddev, int(norm_ones))
        if not h:
            raise RuntimeError("oracle: " + lib().orc_last_error().decode())
        return cls(None, cfg_ints, _handle=h)

    def gen_begin(self, ids: np.ndarray) -> None:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        B, S = ids.shape
        _check(lib().orc_gen_begin(self.h, _p(ids), B, S))
        self.rows = B

    def gen_frame(self, f: int, w: float, temperature: float, top_k: int, masked: bool, seed: int) -> np.ndarray:
        """One frame of generate_tokens (temporal step, rvq_depth x (depth
        step + sampler + feedback)) with Philox draws; returns the frame's ids."""
        out = np.empty(self.depth, np.int32)
        _check(lib().orc_gen_frame(self.h, f, w, temperature, top_k, int(masked), seed, _p(out)))
        return out

    # ---- single-layer probes ----------------------------------------------
    def embed_pe(self, ids: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        B, S = ids.shape
        out = np.empty((B, S, self.d), np.float32)
        _check(lib().orc_embed_pe(self.h, _p(ids), B, S, _p(out)))
        return out

    def encoder_layer(self, layer: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        B, S, _ = x.shape
        out = np.empty_like(x)
        _check(lib().orc_encoder_layer(self.h, layer, _p(x), B, S, _p(out)))
        return out

    def decoder_layer(self, stack: int, layer: int, pos: int, x: np.ndarray) -> np.ndarray:
        """stack 0 = temporal, 1 = depth; writes this step's K/V at `pos`."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        _check(lib().orc_decoder_layer(self.h, stack, layer, pos, _p(x), _p(out)))
        return out

    def get_cache(self, kind: int, layer: int, cap: int):
        """kind 0 temporal self, 1 depth self, 2 cross: (K, V) as (rows, H, cap, 64)."""
        H = self.cfg[4]
        K = np.empty((self.rows, H, cap, 64), np.float32)
        V = np.empty_like(K)
        _check(lib().orc_get_cache(self.h, kind, layer, _p(K), _p(V)))
        return K, V

    def set_cache(self, kind: int, layer: int, K: np.ndarray, V: np.ndarray, enc_len: int) -> None:
        """Overwrite a full-capacity cache (kinds as in get_cache) for
        K.shape[0] rows and an encoder length of enc_len."""
        K = np.ascontiguousarray(K, dtype=np.float32)
        V = np.ascontiguousarray(V, dtype=np.float32)
        _check(lib().orc_set_cache(self.h, kind, layer, _p(K), _p(V), K.shape[0], enc_len))
        self.rows = K.shape[0]

    def lm_head(self, x: np.ndarray, lo: int, hi: int) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty((x.shape[0], hi - lo), np.float32)
        _check(lib().orc_lm_head(self.h, _p(x), x.shape[0], lo, hi, _p(out)))
        return out

    def encode(self, ids: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        B, S = ids.shape
        out = np.empty((B, S, self.d), np.float32)
        _check(lib().orc_encode(self.h, _p(ids), B, S, _p(out)))
        self.rows = B
        return out

    def temporal_step(self, x: Optional[np.ndarray], f: int) -> np.ndarray:
        xin = None if x is None else np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty((self.rows, self.d), np.float32)
        _check(lib().orc_temporal_step(self.h, _p(xin), f, _p(out)))
        return out

    def depth_step(self, x: Optional[np.ndarray], l: int) -> np.ndarray:
        xin = None if x is None else np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty((self.rows, self.V), np.float32)
        _check(lib().orc_depth_step(self.h, _p(xin), l, _p(out)))
        return out

    def generate(self, ids: np.ndarray, num_frames: int, w: float, temperature: float, top_k: int, masked: bool,
                 seed: int, uniforms: Optional[np.ndarray] = None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        B, S = ids.shape
        out = np.empty((num_frames, self.depth), np.int32)
        u = None if uniforms is None else np.ascontiguousarray(uniforms, dtype=np.float32)
        _check(lib().orc_generate(self.h, _p(ids), B, S, num_frames, w, temperature, top_k, int(masked), seed, _p(u),
                                  _p(out)))
        self.rows = B
        return out

    def teacher_forced(self, ids: np.ndarray, tokens: np.ndarray, num_frames: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        B, S = ids.shape
        toks = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        out = np.empty((num_frames, self.depth, B, self.V), np.float32)
        _check(lib().orc_teacher_forced(self.h, _p(ids), B, S, num_frames, _p(toks), _p(out)))
        self.rows = B
        return out

    def close(self):
        if self.h:
            lib().orc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def sample(logits: np.ndarray, level: int, masked: bool, codebook: int, offset: int, w: float, temperature: float,
           top_k: int, uniforms: np.ndarray) -> int:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, V = logits.shape
    u = np.ascontiguousarray(uniforms, dtype=np.float32)
    tok = np.zeros(1, np.int32)
    _check(lib().orc_sample(_p(logits), rows, V, level, int(masked), codebook, offset, w, temperature, top_k, _p(u),
                            _p(tok)))
    return int(tok[0])


def relative_bucket(rel: int, num_buckets: int, max_distance: int) -> int:
    return lib().orc_relative_bucket(rel, num_buckets, max_distance)


def sinusoid(max_length: int, features: int) -> np.ndarray:
    out = np.empty((max_length, features), np.float32)
    lib().orc_sinusoid(max_length, features, _p(out))
    return out


def philox_uniform(seed: int, step: int, idx: int) -> float:
    return lib().orc_philox_uniform(seed, step, idx)


def philox4x32_10(ctr, key):
    c = np.asarray(ctr, np.uint32)
    k = np.asarray(key, np.uint32)
    o = np.zeros(4, np.uint32)
    lib().orc_philox4x32_10(_p(c), _p(k), _p(o))
    return o


def gumbel(u: float) -> float:
    return lib().orc_gumbel(u)


def exact_log(x: float) -> float:
    return lib().orc_exact_log(x)


def cfg_mix(c: float, u: float, w: float) -> float:
    return lib().orc_cfg_mix(c, u, w)


def gelu(x: float, bf16: bool) -> float:
    return lib().orc_gelu(x, int(bf16))


def bf16_round(x: float) -> float:
    return lib().orc_bf16_round(x)


def set_num_threads(n: int):
    lib().orc_set_num_threads(n)


def num_threads() -> int:
    return lib().orc_num_threads()


# ---------------------------------------------------------------------------
# SpectroStream decode phase (oracle/spectrostream_oracle.cpp)
# ---------------------------------------------------------------------------
def _ss_check(rc: int):
    if rc != 0:
        raise RuntimeError("oracle: " + lib().orc_ss_last_error().decode())


class CodecOracle:
    """CPU restatement (float32) of rvq_dequantization, SpectroStreamDecoder
    and istft_postprocess."""

    def __init__(self, decoder_path: str, codebooks_path: str):
        h = lib().orc_ss_create(decoder_path.encode(), codebooks_path.encode())
        if not h:
            raise RuntimeError("oracle: " + lib().orc_ss_last_error().decode())
        self.h = h

    def rvq_dequantize(self, codes: np.ndarray) -> np.ndarray:
        codes = np.ascontiguousarray(codes, dtype=np.int32)
        out = np.empty((codes.shape[0], 256), np.float32)
        _ss_check(lib().orc_ss_dequantize(self.h, codes.ctypes.data, codes.shape[0], codes.shape[1], out.ctypes.data))
        return out

    def decode(self, emb: np.ndarray) -> np.ndarray:
        emb = np.ascontiguousarray(emb, dtype=np.float32)
        B, S, _ = emb.shape
        out = np.empty((B, 4 * S, 480, 4), np.float32)
        _ss_check(lib().orc_ss_decode(self.h, emb.ctypes.data, B, S, out.ctypes.data))
        return out

    def decode_tokens(self, codes: np.ndarray) -> np.ndarray:
        codes = np.ascontiguousarray(codes, dtype=np.int32)
        S, levels = codes.shape
        out = np.empty((S * 1920, 2), np.float32)
        _ss_check(lib().orc_ss_decode_tokens(self.h, codes.ctypes.data, S, levels, out.ctypes.data))
        return out

    def close(self):
        if getattr(self, "h", None):
            lib().orc_ss_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def istft(spec: np.ndarray, target_length: int) -> np.ndarray:
    spec = np.ascontiguousarray(spec, dtype=np.float32)
    B, frames = spec.shape[:2]
    out = np.empty((B, target_length, 2), np.float32)
    _ss_check(lib().orc_ss_istft(spec.ctypes.data, B, frames, target_length, out.ctypes.data))
    return out


def conv2d(x: np.ndarray, w: np.ndarray, b: np.ndarray, stride=(1, 1), causal_pad: bool = False) -> np.ndarray:
    """NHWC x, canonical weight (O, I, kh, kw)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    N, H, W, C = x.shape
    O, I, kh, kw = w.shape
    sh, sw = stride
    if causal_pad:
        ow = -(-W // sw)
        tot = max((ow - 1) * sw + kw - W, 0)
        Hp, Wp = H + kh - sh, W + tot
    else:
        Hp, Wp = H, W
    out = np.empty((N, (Hp - kh) // sh + 1, (Wp - kw) // sw + 1, O), np.float32)
    _ss_check(lib().orc_ss_conv2d(x.ctypes.data, N, H, W, C, w.ctypes.data, b.ctypes.data, O, kh, kw, sh, sw,
                                  int(causal_pad), out.ctypes.data))
    return out


def conv_transpose2d(x: np.ndarray, w: np.ndarray, b: np.ndarray, stride=(1, 1)) -> np.ndarray:
    """NHWC x, canonical weight (I, O, kh, kw)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    N, H, W, C = x.shape
    I, O, kh, kw = w.shape
    sh, sw = stride
    out = np.empty((N, (H - 1) * sh + kh, (W - 1) * sw + kw, O), np.float32)
    _ss_check(lib().orc_ss_conv_transpose2d(x.ctypes.data, N, H, W, C, w.ctypes.data, b.ctypes.data, O, kh, kw, sh,
                                            sw, out.ctypes.data))
    return out


# ---------------------------------------------------------------------------
# MusicCoCa text tower and style-token quantisation (oracle/musiccoca_oracle.cpp)
# ---------------------------------------------------------------------------
class StyleOracle:
    """CPU restatement (float32) of MusicCoCaEncoder::embed_text and of the
    rvq_quantization StyleModel::tokenize applies to its embedding."""

    def __init__(self, encoder_path: str, codebooks_path: str):
        h = lib().orc_mc_create(encoder_path.encode(), codebooks_path.encode())
        if not h:
            raise RuntimeError("oracle: " + lib().orc_mc_last_error().decode())
        self.h = h

    def embed_text(self, ids: np.ndarray, padding: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        pad = np.ascontiguousarray(padding, dtype=np.float32)
        B, L = ids.shape
        out = np.empty((B, 768), np.float32)
        if lib().orc_mc_embed_text(self.h, ids.ctypes.data, pad.ctypes.data, B, L, out.ctypes.data) != 0:
            raise RuntimeError("oracle: " + lib().orc_mc_last_error().decode())
        return out

    def quantize(self, emb: np.ndarray, levels: int) -> np.ndarray:
        emb = np.ascontiguousarray(emb, dtype=np.float32)
        out = np.empty((emb.shape[0], levels), np.int32)
        if lib().orc_mc_quantize(self.h, emb.ctypes.data, emb.shape[0], levels, out.ctypes.data) != 0:
            raise RuntimeError("oracle: " + lib().orc_mc_last_error().decode())
        return out

    def close(self):
        if getattr(self, "h", None):
            lib().orc_mc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

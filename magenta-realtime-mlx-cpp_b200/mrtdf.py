"""Python bindings of libmrtdf.so (include/mrtdf.h) over ctypes.

The names mirror the reference's Depthformer API
(src/magenta_realtime_mlx/depthformer/model.h:72-124, decode.h:48-119):
``Engine`` plays ``Depthformer``, a ``Stream`` owns the KV caches
(``empty_temporal_cache`` / ``empty_depth_cache``) and exposes ``encode``,
``temporal_step``, ``depth_step`` and ``generate_tokens``. Errors raise
``MrtdfError`` with the library's message, where the reference throws.

There is no CPU fallback: importing works without a GPU, but every compute
call goes through the CUDA library and fails loudly when it (or a GPU) is
missing.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libmrtdf.so")

DTYPE_FP32 = 0
DTYPE_BF16 = 1

CONFIG_FIELDS = [
    "vocab_size", "d_model", "d_kv", "d_ff", "num_heads", "num_encoder_layers", "num_temporal_layers",
    "num_depth_layers", "max_encoder_length", "rvq_depth", "temporal_num_buckets", "temporal_max_distance",
    "depth_num_buckets", "depth_max_distance", "codebook_size", "codec_offset", "max_frames", "dtype",
]

# Exported symbols, in include/mrtdf.h order.
EXPORTS = [
    "mrtdf_last_error", "mrtdf_version", "mrtdf_config_preset", "mrtdf_write_random_safetensors", "mrtdf_create",
    "mrtdf_destroy", "mrtdf_load_safetensors", "mrtdf_load_random", "mrtdf_stream_create", "mrtdf_stream_destroy",
    "mrtdf_stream_rows", "mrtdf_encode", "mrtdf_temporal_step", "mrtdf_depth_step", "mrtdf_token_embedding",
    "mrtdf_sample", "mrtdf_sample_noalloc", "mrtdf_generate_tokens", "mrtdf_generate_tokens_dev",
    "mrtdf_teacher_forced_logits", "mrtdf_stream_sync", "mrtdf_stream_cuda", "mrtdf_check_wait_timeout",
    "mrtdf_bench_phases", "mrtdf_bench_l2_read",
    "mrtdf_bench_encoder", "mrtdf_bench_depth", "mrtdf_stream_chunk_kernels", "mrtdf_probe_encoder_layer",
    "mrtdf_probe_set_cache", "mrtdf_probe_decoder_layer", "mrtdf_probe_lm_head", "mrtdf_generate_stream_dev",
    "mrtdf_build_encoder_inputs",
    "mrtdf_context_roll", "mrtdf_llm_to_rvq", "mrtdf_rvq_to_llm", "mrtdf_resolve_inference_bundle",
]


class MrtdfError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[mrtdf status {code}] {msg}")
        self.code = code


PATH_MAX = 4096
BUNDLE_FIELDS = ["spectrostream_encoder", "spectrostream_decoder", "spectrostream_codebooks", "musiccoca_encoder",
                 "musiccoca_codebooks", "musiccoca_vocab", "depthformer"]


class BundlePaths(ctypes.Structure):
    """mrtdf_bundle_paths (include/mrtdf.h): InferenceBundlePaths, weights.h:70-78."""
    _fields_ = [(n, ctypes.c_char * PATH_MAX) for n in BUNDLE_FIELDS]


class Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in CONFIG_FIELDS]

    def as_ints(self):
        return [getattr(self, n) for n in CONFIG_FIELDS]

    def replace(self, **kw) -> "Config":
        c = Config()
        for n in CONFIG_FIELDS:
            setattr(c, n, kw.get(n, getattr(self, n)))
        return c

    @property
    def inner(self) -> int:
        return self.num_heads * self.d_kv


class GenOpts(ctypes.Structure):
    _fields_ = [
        ("num_frames", ctypes.c_int),
        ("rvq_depth", ctypes.c_int),
        ("temperature", ctypes.c_float),
        ("top_k", ctypes.c_int),
        ("guidance_weight", ctypes.c_float),
        ("use_vocab_masks", ctypes.c_int),
        ("seed", ctypes.c_uint64),
        ("uniforms", ctypes.POINTER(ctypes.c_float)),
    ]


_lib = None


def lib() -> ctypes.CDLL:
    """Load libmrtdf.so (build it with magenta-realtime-mlx-cpp_b200/build.py)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise MrtdfError(-1, f"{LIB_PATH} is missing: run magenta-realtime-mlx-cpp_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        L.mrtdf_last_error.restype = ctypes.c_char_p
        L.mrtdf_version.restype = ctypes.c_char_p
        L.mrtdf_stream_cuda.restype = ctypes.c_void_p
        L.mrtdf_stream_cuda.argtypes = [ctypes.c_void_p]
        L.mrtdf_resolve_inference_bundle.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(BundlePaths)]
        L.mrtdf_write_random_safetensors.argtypes = [ctypes.POINTER(Config), ctypes.c_uint64, ctypes.c_float,
                                                     ctypes.c_int, ctypes.c_char_p]
        L.mrtdf_load_random.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_float, ctypes.c_int]
        L.mrtdf_create.argtypes = [ctypes.POINTER(Config), ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]
        L.mrtdf_destroy.argtypes = [ctypes.c_void_p]
        L.mrtdf_load_safetensors.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
        L.mrtdf_stream_create.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_void_p)]
        L.mrtdf_stream_destroy.argtypes = [ctypes.c_void_p]
        L.mrtdf_stream_rows.argtypes = [ctypes.c_void_p]
        L.mrtdf_stream_sync.argtypes = [ctypes.c_void_p]
        for name in ["mrtdf_encode", "mrtdf_temporal_step", "mrtdf_depth_step", "mrtdf_generate_tokens",
                     "mrtdf_generate_tokens_dev", "mrtdf_teacher_forced_logits", "mrtdf_token_embedding",
                     "mrtdf_sample"]:
            getattr(L, name).restype = ctypes.c_int
        L.mrtdf_stream_chunk_kernels.restype = ctypes.c_longlong
        L.mrtdf_stream_chunk_kernels.argtypes = [ctypes.c_void_p]
        L.mrtdf_bench_l2_read.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_double)]
        L.mrtdf_sample_noalloc.restype = ctypes.c_int
        L.mrtdf_sample_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                           ctypes.POINTER(GenOpts), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != 0:
        raise MrtdfError(rc, lib().mrtdf_last_error().decode())


def _fp(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _ip(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))


def preset(name: str, dtype: int = DTYPE_BF16, **overrides) -> Config:
    c = Config()
    _check(lib().mrtdf_config_preset(name.encode(), ctypes.byref(c)))
    c.dtype = dtype
    return c.replace(**overrides) if overrides else c


def write_random_safetensors(cfg: Config, seed: int, path: str, stddev: float = 0.02, norm_ones: bool = True):
    _check(lib().mrtdf_write_random_safetensors(ctypes.byref(cfg), seed, stddev, int(norm_ones), path.encode()))


def gen_opts(cfg: Config, num_frames: int, temperature: float = 1.1, top_k: int = 40, guidance_weight: float = 4.0,
             use_vocab_masks: bool = True, seed: int = 0, uniforms: Optional[np.ndarray] = None) -> GenOpts:
    o = GenOpts()
    o.num_frames = num_frames
    o.rvq_depth = cfg.rvq_depth
    o.temperature = temperature
    o.top_k = top_k
    o.guidance_weight = guidance_weight
    o.use_vocab_masks = int(use_vocab_masks)
    o.seed = seed
    o._uniforms_keepalive = uniforms
    o.uniforms = _fp(uniforms) if uniforms is not None else ctypes.POINTER(ctypes.c_float)()
    return o


class Engine:
    """Depthformer weights on one GPU (Depthformer ctor, model.h:74-75)."""

    def __init__(self, cfg: Config, device: int = 0):
        self.cfg = cfg
        h = ctypes.c_void_p()
        _check(lib().mrtdf_create(ctypes.byref(cfg), device, ctypes.byref(h)))
        self.h = h

    def load_safetensors(self, path: str) -> "Engine":
        _check(lib().mrtdf_load_safetensors(self.h, path.encode()))
        return self

    def load_random(self, seed: int, stddev: float = 0.02, norm_ones: bool = True) -> "Engine":
        _check(lib().mrtdf_load_random(self.h, seed, stddev, int(norm_ones)))
        return self

    def token_embedding(self, ids: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
        out = np.empty((ids.size, self.cfg.d_model), np.float32)
        _check(lib().mrtdf_token_embedding(self.h, _ip(ids), ids.size, _fp(out)))
        return out

    def sample(self, logits: np.ndarray, frame: int, level: int, opts: GenOpts,
               uniforms: Optional[np.ndarray] = None) -> int:
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        rows = logits.shape[0]
        tok = np.zeros(1, np.int32)
        u = None if uniforms is None else np.ascontiguousarray(uniforms, dtype=np.float32)
        _check(lib().mrtdf_sample(self.h, _fp(logits), int(rows == 2), frame, level, ctypes.byref(opts), _fp(u),
                                  _ip(tok)))
        return int(tok[0])

    def sample_noalloc(self, logits_dev_ptr: int, cfg: bool, frame: int, level: int, opts: GenOpts,
                       uniforms_dev_ptr: Optional[int], token_dev_ptr: int, stream: int = 0) -> None:
        """mrtdf_sample on caller-owned device buffers, queued on `stream`
        (a cudaStream_t as int) without waiting; allocates no GPU memory."""
        _check(lib().mrtdf_sample_noalloc(self.h, ctypes.c_void_p(logits_dev_ptr), int(cfg), frame, level,
                                          ctypes.byref(opts), ctypes.c_void_p(uniforms_dev_ptr or None),
                                          ctypes.c_void_p(token_dev_ptr), ctypes.c_void_p(stream or None)))

    def bench_l2_read(self, nbytes: int, reps: int) -> float:
        """GB/s of 16-byte reads over an nbytes buffer held in L2."""
        g = ctypes.c_double()
        _check(lib().mrtdf_bench_l2_read(self.h, ctypes.c_size_t(nbytes), reps, ctypes.byref(g)))
        return g.value

    def bench_encoder(self, rows: int, seq_len: int, reps: int):
        """(ms per encoder pass, algorithmic FLOPs per pass) for `rows`
        sequences of `seq_len` random ids, replayed as one CUDA graph."""
        ms = ctypes.c_float()
        fl = ctypes.c_double()
        _check(lib().mrtdf_bench_encoder(self.h, rows, seq_len, reps, ctypes.byref(ms), ctypes.byref(fl)))
        return ms.value, fl.value

    def close(self):
        if self.h:
            lib().mrtdf_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Stream:
    """A decoding stream: KV arena + step state for `num_sequences` CFG pairs."""

    def __init__(self, engine: Engine, num_sequences: int = 1, cfg: bool = True):
        self.engine = engine
        self.cfg = engine.cfg
        h = ctypes.c_void_p()
        _check(lib().mrtdf_stream_create(engine.h, num_sequences, int(cfg), ctypes.byref(h)))
        self.h = h
        self.num_sequences = num_sequences
        self.rows = lib().mrtdf_stream_rows(h)

    def encode(self, ids: np.ndarray, want_output: bool = False) -> Optional[np.ndarray]:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        S = ids.shape[-1]
        out = np.empty((self.rows, S, self.cfg.d_model), np.float32) if want_output else None
        _check(lib().mrtdf_encode(self.h, _ip(ids), S, _fp(out)))
        return out

    def temporal_step(self, x: Optional[np.ndarray], frame_idx: int) -> np.ndarray:
        xin = None if x is None else np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty((self.rows, self.cfg.d_model), np.float32)
        _check(lib().mrtdf_temporal_step(self.h, _fp(xin), frame_idx, _fp(out)))
        return out

    def depth_step(self, x: Optional[np.ndarray], depth_idx: int) -> np.ndarray:
        xin = None if x is None else np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty((self.rows, self.cfg.vocab_size), np.float32)
        _check(lib().mrtdf_depth_step(self.h, _fp(xin), depth_idx, _fp(out)))
        return out

    def generate_tokens(self, ids: np.ndarray, opts: GenOpts, seeds: Optional[Sequence[int]] = None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        S = ids.shape[-1]
        out = np.empty((self.num_sequences, opts.num_frames, self.cfg.rvq_depth), np.int32)
        sd = None
        if seeds is not None:
            sd = (ctypes.c_uint64 * self.num_sequences)(*seeds)
        _check(lib().mrtdf_generate_tokens(self.h, _ip(ids), S, ctypes.byref(opts), sd, _ip(out)))
        return out

    def generate_tokens_dev(self, ids_dev_ptr: int, seq_len: int, opts: GenOpts, out_dev_ptr: int,
                            seeds: Optional[Sequence[int]] = None) -> None:
        sd = None
        if seeds is not None:
            sd = (ctypes.c_uint64 * self.num_sequences)(*seeds)
        _check(lib().mrtdf_generate_tokens_dev(self.h, ctypes.c_void_p(ids_dev_ptr), seq_len, ctypes.byref(opts), sd,
                                               ctypes.c_void_p(out_dev_ptr)))

    def generate_stream_dev(self, context_dev_ptr: int, ctx_frames: int, enc_depth: int, style_dev_ptr: int,
                            style_depth: int, num_chunks: int, opts: GenOpts, out_dev_ptr: int,
                            seeds: Optional[Sequence[int]] = None) -> None:
        """num_chunks streaming chunks on the device (context rolled in place);
        returns once queued."""
        sd = None
        if seeds is not None:
            sd = (ctypes.c_uint64 * (num_chunks * self.num_sequences))(*seeds)
        _check(lib().mrtdf_generate_stream_dev(self.h, ctypes.c_void_p(context_dev_ptr), ctx_frames, enc_depth,
                                               ctypes.c_void_p(style_dev_ptr), style_depth, num_chunks,
                                               ctypes.byref(opts), sd, ctypes.c_void_p(out_dev_ptr)))

    def teacher_forced_logits(self, ids: np.ndarray, tokens: np.ndarray, num_frames: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        toks = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        out = np.empty((num_frames, self.cfg.rvq_depth, self.rows, self.cfg.vocab_size), np.float32)
        _check(lib().mrtdf_teacher_forced_logits(self.h, _ip(ids), ids.shape[-1], _ip(toks), num_frames, _fp(out)))
        return out

    def sync(self) -> None:
        _check(lib().mrtdf_stream_sync(self.h))

    def check_wait_timeout(self, timeout_us: int) -> None:
        """Queue a device wait that nothing completes, bounded by timeout_us;
        raises MrtdfError with MRTDF_ERR_TIMEOUT (6) when it gives up."""
        _check(lib().mrtdf_check_wait_timeout(self.h, timeout_us))

    def chunk_kernels(self) -> int:
        """Kernel nodes of the last chunk's CUDA graph (-1: no graph)."""
        return int(lib().mrtdf_stream_chunk_kernels(self.h))

    def bench_depth(self, opts: GenOpts, frames: int, reps: int):
        """(us per depth step, algorithmic bytes per step, launches per step)
        of frames x rvq_depth depth steps from N(0, 1) hidden states."""
        us = ctypes.c_float()
        b = ctypes.c_double()
        n = ctypes.c_longlong()
        _check(lib().mrtdf_bench_depth(self.h, ctypes.byref(opts), frames, reps, ctypes.byref(us), ctypes.byref(b),
                                       ctypes.byref(n)))
        return us.value, b.value, n.value

    def bench_phases(self, opts: GenOpts, stack_mask: int, reps: int):
        """(ms per chunk replay, launches, algorithmic bytes) of the
        weight-streaming decode launches of one chunk for the stacks in
        stack_mask (1 temporal, 2 depth + lm_head, 3 both), CUDA events on
        this stream."""
        ms = ctypes.c_float()
        n = ctypes.c_longlong()
        b = ctypes.c_double()
        _check(lib().mrtdf_bench_phases(self.h, ctypes.byref(opts), stack_mask, reps, ctypes.byref(ms),
                                        ctypes.byref(n), ctypes.byref(b)))
        return ms.value, n.value, b.value

    def cuda_stream(self) -> int:
        return lib().mrtdf_stream_cuda(self.h)

    # ---- single-layer probes (one step of the production launch sequence) ----
    def probe_encoder_layer(self, layer: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        _check(lib().mrtdf_probe_encoder_layer(self.h, layer, _fp(x), x.shape[1], _fp(out)))
        return out

    def probe_set_cache(self, kind: int, layer: int, k: np.ndarray, v: np.ndarray) -> None:
        """kind 0 temporal self, 1 depth self, 2 cross; k / v (rows, H, len, 64)."""
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        _check(lib().mrtdf_probe_set_cache(self.h, kind, layer, _fp(k), _fp(v), k.shape[2]))

    def probe_decoder_layer(self, stack: int, layer: int, pos: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        _check(lib().mrtdf_probe_decoder_layer(self.h, stack, layer, pos, _fp(x), _fp(out)))
        return out

    def probe_lm_head(self, level: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        n = self.cfg.codebook_size if level >= 0 else self.cfg.vocab_size
        out = np.empty((x.shape[0], n), np.float32)
        _check(lib().mrtdf_probe_lm_head(self.h, level, _fp(x), _fp(out)))
        return out

    def close(self):
        if self.h:
            lib().mrtdf_stream_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- streaming glue (System, system.cpp) -----------------------------------
def build_encoder_inputs(context: np.ndarray, style: np.ndarray, enc_depth: int, codebook_size: int,
                         codec_offset: int) -> np.ndarray:
    context = np.ascontiguousarray(context, dtype=np.int32)
    style = np.ascontiguousarray(style, dtype=np.int32)
    F, D = context.shape
    out = np.empty((2, F * enc_depth + style.size), np.int32)
    _check(lib().mrtdf_build_encoder_inputs(_ip(context), F, D, enc_depth, _ip(style), style.size, codebook_size,
                                            codec_offset, _ip(out)))
    return out


def context_roll(context: np.ndarray, new_codes: np.ndarray) -> np.ndarray:
    ctx = np.array(context, dtype=np.int32, copy=True, order="C")
    new = np.ascontiguousarray(new_codes, dtype=np.int32)
    _check(lib().mrtdf_context_roll(_ip(ctx), ctx.shape[0], ctx.shape[1], _ip(new), new.shape[0]))
    return ctx


def llm_to_rvq(tokens: np.ndarray, codebook_size: int, codec_offset: int) -> np.ndarray:
    t = np.ascontiguousarray(tokens, dtype=np.int32)
    out = np.empty_like(t)
    _check(lib().mrtdf_llm_to_rvq(_ip(t), t.shape[0], t.shape[1], codebook_size, codec_offset, _ip(out)))
    return out


def resolve_inference_bundle(cache_root: str, tag: str) -> dict:
    """resolve_inference_bundle (weights.cpp:72-120): {field: path} of the
    seven bundle files; MrtdfError (MRTDF_ERR_IO) when the root is not a
    directory or a file is missing."""
    out = BundlePaths()
    _check(lib().mrtdf_resolve_inference_bundle(str(cache_root).encode(), tag.encode(), ctypes.byref(out)))
    return {n: getattr(out, n).decode() for n in BUNDLE_FIELDS}


def rvq_to_llm(tokens: np.ndarray, codebook_size: int, codec_offset: int) -> np.ndarray:
    t = np.ascontiguousarray(tokens, dtype=np.int32)
    out = np.empty_like(t)
    _check(lib().mrtdf_rvq_to_llm(_ip(t), t.shape[0], t.shape[1], codebook_size, codec_offset, _ip(out)))
    return out

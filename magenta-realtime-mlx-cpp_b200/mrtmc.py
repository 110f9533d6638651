"""Python bindings of the style path (include/mrtmc.h) over ctypes, in the
same library as mrtdf.py.

The names mirror the reference (src/magenta_realtime_mlx/musiccoca.h,
style_model.h, rvq.h): ``StyleModel.embed_text`` plays
``MusicCoCaEncoder::embed_text``, ``StyleModel.quantize`` plays
``rvq_quantization`` (``StyleModel::tokenize`` with 12 levels) and
``StyleModel.style_tokens_lm`` plays ``StyleModel::style_tokens_lm`` after
its SentencePiece step (the caller passes the token ids and padding mask).
Errors raise ``mrtdf.MrtdfError``. There is no CPU fallback.
"""
from __future__ import annotations

import ctypes

import numpy as np

import mrtdf

EMBED_DIM = 768
MAX_TEXT_LEN = 128
RVQ_DEPTH = 12

# Exported symbols, in include/mrtmc.h order.
EXPORTS = [
    "mrtmc_create", "mrtmc_destroy", "mrtmc_load_safetensors", "mrtmc_embed_text", "mrtmc_quantize",
    "mrtmc_style_tokens", "mrtmc_cuda_stream", "mrtmc_embed_kernels",
]

_bound = False


def lib() -> ctypes.CDLL:
    global _bound
    L = mrtdf.lib()
    if not _bound:
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p
        L.mrtmc_create.argtypes = [I, I, ctypes.POINTER(P)]
        L.mrtmc_destroy.argtypes = [P]
        L.mrtmc_destroy.restype = None
        L.mrtmc_load_safetensors.argtypes = [P, F, F]
        L.mrtmc_embed_text.argtypes = [P, P, P, I, I, P]
        L.mrtmc_quantize.argtypes = [P, P, I, I, P]
        L.mrtmc_style_tokens.argtypes = [P, P, P, I, I, I, I, I, P]
        L.mrtmc_cuda_stream.argtypes = [P]
        L.mrtmc_cuda_stream.restype = P
        L.mrtmc_embed_kernels.argtypes = [P, I, I]
        L.mrtmc_embed_kernels.restype = ctypes.c_longlong
        _bound = True
    return L


def _check(rc: int) -> None:
    mrtdf._check(rc)


def write_random_safetensors(encoder_path: str, codebooks_path: str, seed: int = 0, vocab: int = 64000,
                             levels: int = RVQ_DEPTH, codebook_size: int = 1024) -> None:
    """A random-init text-tower bundle with the reference's key layout
    (musiccoca.cpp constructors: token_embedding, text_layers.{0..11},
    text_exit_ln, text_pooler) and a (levels, codebook_size, 768) codebook
    bundle: weights N(0, 1 / fan_in), biases N(0, 0.02^2), LayerNorm scales
    1 + N(0, 0.1^2) and shifts N(0, 0.1^2), numpy seed `seed`. No reference
    counterpart (the real bundles are downloaded; none is available here)."""
    from safetensors.numpy import save_file

    D, H, DH, FF, POOL_DH = EMBED_DIM, 12, 64, 3072, 256
    rng = np.random.default_rng(seed)
    w = {}

    def lin(p, out, inp):
        w[p + ".weight"] = (rng.standard_normal((out, inp), dtype=np.float32) / np.float32(np.sqrt(inp)))
        w[p + ".bias"] = rng.standard_normal(out, dtype=np.float32) * np.float32(0.02)

    def ln(p):
        w[p + ".weight"] = 1 + np.float32(0.1) * rng.standard_normal(D, dtype=np.float32)
        w[p + ".bias"] = np.float32(0.1) * rng.standard_normal(D, dtype=np.float32)

    w["token_embedding.weight"] = rng.standard_normal((vocab, D), dtype=np.float32) / np.float32(np.sqrt(D))
    for i in range(12):
        p = f"text_layers.{i}"
        ln(p + ".attn_ln")
        ln(p + ".ffn_ln")
        for n in ("q", "k", "v"):
            lin(f"{p}.attn.{n}_proj", H * DH, D)
        lin(p + ".attn.o_proj", D, H * DH)
        lin(p + ".ffn_w1", FF, D)
        lin(p + ".ffn_w2", D, FF)
    ln("text_exit_ln")
    ln("text_pooler.ln")
    w["text_pooler.query"] = rng.standard_normal((1, 1, D), dtype=np.float32)
    for n in ("q", "k", "v"):
        lin(f"text_pooler.attn.{n}_proj", H * POOL_DH, D)
    lin("text_pooler.attn.o_proj", D, H * POOL_DH)
    w["text_pooler.attn._per_dim_scale"] = np.float32(0.5) * rng.standard_normal(POOL_DH, dtype=np.float32)
    save_file(w, encoder_path)
    cb = rng.standard_normal((levels, codebook_size, D), dtype=np.float32) / np.float32(np.sqrt(D))
    save_file({"codebooks": cb}, codebooks_path)


class StyleModel:
    """MusicCoCa text tower + style RVQ on one GPU, for up to ``max_batch``
    prompts of up to 128 tokens per call."""

    def __init__(self, max_batch: int = 1, device: int = 0):
        h = ctypes.c_void_p()
        _check(lib().mrtmc_create(device, max_batch, ctypes.byref(h)))
        self.h = h
        self.max_batch = max_batch

    def load_safetensors(self, encoder_path: str, codebooks_path: str) -> "StyleModel":
        _check(lib().mrtmc_load_safetensors(self.h, encoder_path.encode(), codebooks_path.encode()))
        return self

    def embed_text(self, ids: np.ndarray, pad: np.ndarray) -> np.ndarray:
        """ids (B, L) int32, pad (B, L) float (1.0 = padding) -> (B, 768)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        pad = np.ascontiguousarray(pad, dtype=np.float32)
        if ids.ndim != 2 or pad.shape != ids.shape:
            raise mrtdf.MrtdfError(1, "embed_text: token_ids and padding_mask must be (B, L)")
        B, L = ids.shape
        out = np.empty((B, EMBED_DIM), np.float32)
        _check(lib().mrtmc_embed_text(self.h, ids.ctypes.data, pad.ctypes.data, B, L, out.ctypes.data))
        return out

    def quantize(self, emb: np.ndarray, levels: int = RVQ_DEPTH) -> np.ndarray:
        """emb (N, 768) -> tokens (N, levels) int32."""
        emb = np.ascontiguousarray(emb, dtype=np.float32)
        if emb.ndim != 2 or emb.shape[1] != EMBED_DIM:
            raise mrtdf.MrtdfError(1, "rvq_quantization: vectors must be (N, 768)")
        out = np.empty((emb.shape[0], levels), np.int32)
        _check(lib().mrtmc_quantize(self.h, emb.ctypes.data, emb.shape[0], levels, out.ctypes.data))
        return out

    def style_tokens_lm(self, ids: np.ndarray, pad: np.ndarray, encoder_style_rvq_depth: int = 6,
                        style_rvq_codebook_size: int = 1024, vocab_style_offset: int = 17410) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        pad = np.ascontiguousarray(pad, dtype=np.float32)
        if ids.ndim != 2 or pad.shape != ids.shape:
            raise mrtdf.MrtdfError(1, "style_tokens_lm: token_ids and padding_mask must be (B, L)")
        B, L = ids.shape
        out = np.empty((B, encoder_style_rvq_depth), np.int32)
        _check(lib().mrtmc_style_tokens(self.h, ids.ctypes.data, pad.ctypes.data, B, L, encoder_style_rvq_depth,
                                        style_rvq_codebook_size, vocab_style_offset, out.ctypes.data))
        return out

    def embed_kernels(self, B: int, L: int) -> int:
        return int(lib().mrtmc_embed_kernels(self.h, B, L))

    def cuda_stream(self) -> int:
        return int(lib().mrtmc_cuda_stream(self.h) or 0)

    def close(self) -> None:
        if self.h:
            lib().mrtmc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

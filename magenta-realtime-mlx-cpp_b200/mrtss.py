"""Python bindings of the SpectroStream decode phase (include/mrtss.h) over
ctypes, in the same library as mrtdf.py.

The names mirror the reference (src/magenta_realtime_mlx/spectrostream.h,
rvq.h): ``Codec.decode`` plays ``SpectroStreamDecoder::operator()``,
``Codec.istft`` plays ``istft_postprocess``, ``Codec.rvq_dequantize`` plays
``rvq_dequantization`` and ``Codec.decode_tokens`` is the codec block of
``System::generate_chunk`` (system.cpp:372-390). Errors raise
``mrtdf.MrtdfError``. There is no CPU fallback.
"""
from __future__ import annotations

import ctypes

import numpy as np

import mrtdf

EMBED_DIM = 256
STFT_BINS = 480
FRAME_SAMPLES = 1920

# Exported symbols, in include/mrtss.h order.
EXPORTS = [
    "mrtss_write_random_safetensors", "mrtss_create", "mrtss_destroy", "mrtss_load_safetensors", "mrtss_load_random",
    "mrtss_rvq_dequantize", "mrtss_decode", "mrtss_istft", "mrtss_decode_tokens", "mrtss_decode_tokens_dev",
    "mrtss_sync", "mrtss_cuda_stream", "mrtss_decode_kernels",
]

_bound = False


def lib() -> ctypes.CDLL:
    global _bound
    L = mrtdf.lib()
    if not _bound:
        P, I, U64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_char_p
        L.mrtss_write_random_safetensors.argtypes = [U64, I, F, F]
        L.mrtss_create.argtypes = [I, I, I, ctypes.POINTER(P)]
        L.mrtss_destroy.argtypes = [P]
        L.mrtss_destroy.restype = None
        L.mrtss_load_safetensors.argtypes = [P, F, F]
        L.mrtss_load_random.argtypes = [P, U64, I]
        L.mrtss_rvq_dequantize.argtypes = [P, P, I, I, P]
        L.mrtss_decode.argtypes = [P, P, I, I, P]
        L.mrtss_istft.argtypes = [P, P, I, I, I, P]
        L.mrtss_decode_tokens.argtypes = [P, P, I, I, I, P]
        L.mrtss_decode_tokens_dev.argtypes = [P, P, I, I, I, P]
        L.mrtss_sync.argtypes = [P]
        L.mrtss_cuda_stream.argtypes = [P]
        L.mrtss_cuda_stream.restype = P
        L.mrtss_decode_kernels.argtypes = [P, I, I]
        L.mrtss_decode_kernels.restype = ctypes.c_longlong
        _bound = True
    return L


def _check(rc: int) -> None:
    mrtdf._check(rc)


def write_random_safetensors(seed: int, levels: int, decoder_path: str, codebooks_path: str) -> None:
    _check(lib().mrtss_write_random_safetensors(seed, levels, decoder_path.encode(), codebooks_path.encode()))


class Codec:
    """SpectroStream decoder + iSTFT on one GPU, for up to ``max_batch``
    sequences of up to ``max_frames`` codec frames per call."""

    def __init__(self, max_batch: int = 1, max_frames: int = 51, device: int = 0):
        h = ctypes.c_void_p()
        _check(lib().mrtss_create(device, max_batch, max_frames, ctypes.byref(h)))
        self.h = h
        self.max_batch, self.max_frames = max_batch, max_frames

    def load_safetensors(self, decoder_path: str, codebooks_path: str) -> "Codec":
        _check(lib().mrtss_load_safetensors(self.h, decoder_path.encode(), codebooks_path.encode()))
        return self

    def load_random(self, seed: int, levels: int = 16) -> "Codec":
        _check(lib().mrtss_load_random(self.h, seed, levels))
        return self

    def rvq_dequantize(self, codes: np.ndarray) -> np.ndarray:
        codes = np.ascontiguousarray(codes, dtype=np.int32)
        n, levels = codes.shape
        out = np.empty((n, EMBED_DIM), np.float32)
        _check(lib().mrtss_rvq_dequantize(self.h, codes.ctypes.data, n, levels, out.ctypes.data))
        return out

    def decode(self, embeddings: np.ndarray) -> np.ndarray:
        emb = np.ascontiguousarray(embeddings, dtype=np.float32)
        B, S, D = emb.shape
        if D != EMBED_DIM:
            raise mrtdf.MrtdfError(1, "SpectroStreamDecoder: embeddings must be (B, S, 256)")
        out = np.empty((B, 4 * S, STFT_BINS, 4), np.float32)
        _check(lib().mrtss_decode(self.h, emb.ctypes.data, B, S, out.ctypes.data))
        return out

    def istft(self, spec: np.ndarray, target_length: int) -> np.ndarray:
        spec = np.ascontiguousarray(spec, dtype=np.float32)
        B, frames = spec.shape[:2]
        out = np.empty((B, target_length, 2), np.float32)
        _check(lib().mrtss_istft(self.h, spec.ctypes.data, B, frames, target_length, out.ctypes.data))
        return out

    def decode_tokens(self, codes: np.ndarray) -> np.ndarray:
        """codes (B, S, levels) or (S, levels) -> audio (B, S * 1920, 2)."""
        codes = np.ascontiguousarray(codes, dtype=np.int32)
        squeeze = codes.ndim == 2
        if squeeze:
            codes = codes[None]
        B, S, levels = codes.shape
        out = np.empty((B, S * FRAME_SAMPLES, 2), np.float32)
        _check(lib().mrtss_decode_tokens(self.h, codes.ctypes.data, B, S, levels, out.ctypes.data))
        return out[0] if squeeze else out

    def decode_tokens_dev(self, codes_dev_ptr: int, B: int, S: int, levels: int, audio_dev_ptr: int) -> None:
        _check(lib().mrtss_decode_tokens_dev(self.h, codes_dev_ptr, B, S, levels, audio_dev_ptr))

    def sync(self) -> None:
        _check(lib().mrtss_sync(self.h))

    def cuda_stream(self) -> int:
        return lib().mrtss_cuda_stream(self.h)

    def decode_kernels(self, B: int, S: int) -> int:
        return int(lib().mrtss_decode_kernels(self.h, B, S))

    def close(self):
        if getattr(self, "h", None):
            lib().mrtss_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

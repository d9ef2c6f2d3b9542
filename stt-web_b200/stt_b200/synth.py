"""Seeded synthetic checkpoints and audio-token streams (no download needed).

Thin wrappers over stt_synth_* in libsttb200; the generator itself is C++ (csrc/synth.cpp).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import GGML_BF16, check, lib, stt_synth_params


@dataclass
class SynthSpec:
    seed: int = 0x5EED5EED
    num_layers: int = 16
    hidden_size: int = 2048
    num_heads: int = 16
    ffn_hidden: int = 8448
    vocab_size: int = 8000
    text_in_vocab_size: int = 8001
    num_codebooks: int = 32
    audio_vocab_size: int = 2049
    embedding_dtype: int = GGML_BF16
    weight_std: float = 0.02
    norm_mean: float = 1.0
    norm_std: float = 0.02
    n_threads: int = 0

    def to_c(self) -> stt_synth_params:
        p = stt_synth_params()
        for k, v in self.__dict__.items():
            setattr(p, k, v)
        return p


class GgufBuffer:
    """A GGUF file in library-owned host memory; `.array` views it without copying."""

    def __init__(self, ptr, length):
        self._ptr = ptr
        self.length = length
        self.array = np.ctypeslib.as_array(ptr, shape=(length,))

    @property
    def address(self) -> int:
        return C.cast(self._ptr, C.c_void_p).value

    def close(self):
        if self._ptr:
            self.array = None
            lib().stt_synth_free(self._ptr)
            self._ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def synth_gguf(spec: SynthSpec | None = None) -> GgufBuffer:
    spec = spec or SynthSpec()
    p = spec.to_c()
    ptr = C.POINTER(C.c_uint8)()
    n = C.c_size_t()
    check(lib().stt_synth_gguf(C.byref(p), C.byref(ptr), C.byref(n)), "stt_synth_gguf")
    return GgufBuffer(ptr, n.value)


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32).ravel())
    out = np.empty(a.size // 32 * 18, dtype=np.uint8)
    check(lib().stt_synth_quantize_q4_0(a.ctypes.data_as(C.POINTER(C.c_float)), a.size,
                                        out.ctypes.data_as(C.POINTER(C.c_uint8))), "stt_synth_quantize_q4_0")
    return out


def audio_tokens(seed: int, stream: int, n_frames: int, first_frame: int = 0, num_codebooks: int = 32) -> np.ndarray:
    out = np.empty((n_frames, num_codebooks), dtype=np.uint32)
    check(lib().stt_synth_audio_tokens(seed, stream, first_frame, n_frames, num_codebooks,
                                       out.ctypes.data_as(C.POINTER(C.c_uint32))), "stt_synth_audio_tokens")
    return out

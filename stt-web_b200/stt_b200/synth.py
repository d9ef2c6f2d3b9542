"""Seeded synthetic checkpoints and audio-token streams (no download needed).

Thin wrappers over the stt_synth_* calls of libsttsynth.so (include/stt_synth.h), a host-only
library built beside libsttb200.so from csrc/synth.cpp.  Loading this module never loads the
decode library, so a CPU-only program can generate the same checkpoint bytes.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
# The generator library this module loads (on first use).  A program that must not map anything of
# the decode package (the CPU baseline) points it at another build of the same source first.
SYNTH_LIB_PATH = os.path.join(_HERE, "libsttsynth.so")

GGML_F32, GGML_Q4_0, GGML_BF16 = 0, 2, 30


class stt_synth_params(C.Structure):
    _fields_ = [
        ("seed", C.c_uint64),
        ("num_layers", C.c_int32),
        ("hidden_size", C.c_int32),
        ("num_heads", C.c_int32),
        ("ffn_hidden", C.c_int32),
        ("vocab_size", C.c_int32),
        ("text_in_vocab_size", C.c_int32),
        ("num_codebooks", C.c_int32),
        ("audio_vocab_size", C.c_int32),
        ("embedding_dtype", C.c_int32),
        ("weight_std", C.c_float),
        ("norm_mean", C.c_float),
        ("norm_std", C.c_float),
        ("n_threads", C.c_int32),
    ]


_U8P = C.POINTER(C.c_uint8)
# name -> (restype, argtypes); every symbol declared in include/stt_synth.h
SYNTH_SIGNATURES = {
    "stt_synth_default": (None, [C.POINTER(stt_synth_params)]),
    "stt_synth_gguf": (C.c_int, [C.POINTER(stt_synth_params), C.POINTER(_U8P), C.POINTER(C.c_size_t)]),
    "stt_synth_free": (None, [_U8P]),
    "stt_synth_quantize_q4_0": (C.c_int, [C.POINTER(C.c_float), C.c_size_t, _U8P]),
    "stt_synth_audio_tokens": (C.c_int, [C.c_uint64, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                         C.POINTER(C.c_uint32)]),
    "stt_synth_last_error": (C.c_char_p, []),
}

_slib = None


def synth_lib() -> C.CDLL:
    """Loads libsttsynth.so once; raises if it has not been built."""
    global _slib
    if _slib is None:
        if not os.path.exists(SYNTH_LIB_PATH):
            raise RuntimeError(f"{SYNTH_LIB_PATH} is missing: build it with `make -C stt-web_b200`")
        L = C.CDLL(SYNTH_LIB_PATH)
        for name, (res, args) in SYNTH_SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _slib = L
    return _slib


class SynthError(RuntimeError):
    def __init__(self, code: int, where: str):
        msg = synth_lib().stt_synth_last_error().decode("utf-8", "replace")
        super().__init__(f"{where}: status {code}: {msg}")
        self.code = code


def _check(code: int, where: str) -> None:
    if code != 0:
        raise SynthError(code, where)


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
            synth_lib().stt_synth_free(self._ptr)
            self._ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def synth_gguf(spec: SynthSpec | None = None) -> GgufBuffer:
    spec = spec or SynthSpec()
    p = spec.to_c()
    ptr = _U8P()
    n = C.c_size_t()
    _check(synth_lib().stt_synth_gguf(C.byref(p), C.byref(ptr), C.byref(n)), "stt_synth_gguf")
    return GgufBuffer(ptr, n.value)


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32).ravel())
    out = np.empty(a.size // 32 * 18, dtype=np.uint8)
    _check(synth_lib().stt_synth_quantize_q4_0(a.ctypes.data_as(C.POINTER(C.c_float)), a.size,
                                               out.ctypes.data_as(_U8P)), "stt_synth_quantize_q4_0")
    return out


def audio_tokens(seed: int, stream: int, n_frames: int, first_frame: int = 0, num_codebooks: int = 32) -> np.ndarray:
    out = np.empty((n_frames, num_codebooks), dtype=np.uint32)
    _check(synth_lib().stt_synth_audio_tokens(seed, stream, first_frame, n_frames, num_codebooks,
                                              out.ctypes.data_as(C.POINTER(C.c_uint32))), "stt_synth_audio_tokens")
    return out

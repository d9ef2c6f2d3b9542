"""ctypes wrapper of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the CPU-baseline leg
of bench.py, as the checker.  The library under test never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")

KV_BF16 = 1
GEMM_BF16 = 2


class orc_config(C.Structure):
    _fields_ = [
        ("num_layers", C.c_int32),
        ("num_heads", C.c_int32),
        ("num_codebooks", C.c_int32),
        ("text_delay", C.c_int32),
        ("max_seq_len", C.c_int32),
        ("sliding_window", C.c_int32),
        ("rope_theta", C.c_double),
        ("text_padding_id", C.c_uint32),
        ("text_start_token", C.c_uint32),
    ]


_lib = None


def build() -> None:
    subprocess.check_call(["make", "-s", "-C", HERE], stdout=subprocess.DEVNULL)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = C.CDLL(LIB)
        P, U8P, U32P, F32P = C.c_void_p, C.POINTER(C.c_uint8), C.POINTER(C.c_uint32), C.POINTER(C.c_float)
        L.orc_config_default.argtypes = [C.POINTER(orc_config)]
        L.orc_f16_to_f32_gguf.restype = C.c_float
        L.orc_f16_to_f32_gguf.argtypes = [C.c_uint16]
        L.orc_f16_to_f32_ieee.restype = C.c_float
        L.orc_f16_to_f32_ieee.argtypes = [C.c_uint16]
        L.orc_quantize_q4_0.argtypes = [F32P, C.c_size_t, U8P]
        L.orc_dequant_q4_0.argtypes = [U8P, C.c_int64, C.c_int64, F32P]
        L.orc_embed_id_add_q4.argtypes = [U8P, C.c_int64, C.c_uint32, F32P]
        L.orc_q4_matmul.argtypes = [U8P, C.c_int64, C.c_int64, F32P, C.c_int64, F32P, C.c_uint32]
        L.orc_model_load.restype = C.c_int
        L.orc_model_load.argtypes = [U8P, C.c_size_t, C.POINTER(orc_config), C.POINTER(P)]
        L.orc_model_free.argtypes = [P]
        L.orc_model_dims.argtypes = [P] + [C.POINTER(C.c_int32)] * 4
        L.orc_stream_new.restype = P
        L.orc_stream_new.argtypes = [P, C.c_uint32]
        L.orc_stream_free.argtypes = [P]
        L.orc_stream_reset.argtypes = [P]
        L.orc_forward.restype = C.c_int64
        L.orc_forward.argtypes = [P, U32P, C.c_uint32, F32P]
        L.orc_feed_frame.restype = C.c_int64
        L.orc_feed_frame.argtypes = [P, U32P]
        I64P = C.POINTER(C.c_int64)
        L.orc_forward_batch.restype = C.c_int
        L.orc_forward_batch.argtypes = [C.POINTER(P), C.c_int, U32P, U32P, F32P, I64P]
        L.orc_feed_frame_batch.restype = C.c_int
        L.orc_feed_frame_batch.argtypes = [C.POINTER(P), C.c_int, U32P, F32P, I64P]
        L.orc_forward_gpu_token.restype = C.c_int64
        L.orc_forward_gpu_token.argtypes = [P, U32P, C.c_int, C.c_uint32, C.c_uint32, F32P]
        L.orc_flush.restype = C.c_int
        L.orc_flush.argtypes = [P, U32P, C.c_int]
        L.orc_stream_state.argtypes = [P, C.POINTER(C.c_int64)]
        L.orc_stream_set_last_text_token.argtypes = [P, C.c_uint32]
        L.orc_stream_set_delay_state.argtypes = [P, C.c_uint32, C.c_uint32, C.c_uint32]
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_get_threads.restype = C.c_int
        L.orc_last_error.restype = C.c_char_p
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(C.POINTER(t))


def f16_to_f32_gguf(bits: int) -> float:
    return lib().orc_f16_to_f32_gguf(bits)


def f16_to_f32_ieee(bits: int) -> float:
    return lib().orc_f16_to_f32_ieee(bits)


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32).ravel())
    out = np.empty(a.size // 32 * 18, dtype=np.uint8)
    lib().orc_quantize_q4_0(_p(a, C.c_float), a.size, _p(out, C.c_uint8))
    return out


def dequant_q4_0(raw: np.ndarray, rows: int, k: int) -> np.ndarray:
    r = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty((rows, k), dtype=np.float32)
    lib().orc_dequant_q4_0(_p(r, C.c_uint8), rows, k, _p(out, C.c_float))
    return out


def embed_id_add_q4(table: np.ndarray, dim: int, token: int, out: np.ndarray) -> None:
    t = np.ascontiguousarray(table, dtype=np.uint8)
    assert out.dtype == np.float32 and out.flags.c_contiguous
    lib().orc_embed_id_add_q4(_p(t, C.c_uint8), dim, token, _p(out, C.c_float))


def q4_matmul(raw: np.ndarray, n: int, k: int, x: np.ndarray, flags: int = 0) -> np.ndarray:
    w = np.ascontiguousarray(raw, dtype=np.uint8)
    xx = np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1, k))
    out = np.empty((xx.shape[0], n), dtype=np.float32)
    lib().orc_q4_matmul(_p(w, C.c_uint8), n, k, _p(xx, C.c_float), xx.shape[0], _p(out, C.c_float), flags)
    return out


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


def get_threads() -> int:
    return lib().orc_get_threads()


class OracleModel:
    """orc_model over a GGUF buffer that must stay alive (kept referenced here)."""

    def __init__(self, gguf: np.ndarray, text_delay: int = 6, text_start_token: int = 8000,
                 max_seq_len: int = 4096, sliding_window: int = 750, num_layers: int = 16, num_heads: int = 16,
                 num_codebooks: int = 32):
        self._buf = gguf
        cfg = orc_config()
        lib().orc_config_default(C.byref(cfg))
        cfg.text_delay, cfg.text_start_token = text_delay, text_start_token
        cfg.max_seq_len, cfg.sliding_window = max_seq_len, sliding_window
        cfg.num_layers, cfg.num_heads, cfg.num_codebooks = num_layers, num_heads, num_codebooks
        self.cfg = cfg
        h = C.c_void_p()
        rc = lib().orc_model_load(_p(gguf, C.c_uint8), gguf.size, C.byref(cfg), C.byref(h))
        if rc != 0:
            raise RuntimeError("oracle load failed: " + lib().orc_last_error().decode())
        self._h = h
        d = [C.c_int32() for _ in range(4)]
        lib().orc_model_dims(self._h, *[C.byref(x) for x in d])
        self.hidden, self.ffn, self.vocab, self.text_vocab = [x.value for x in d]

    def stream(self, flags: int = 0) -> "OracleStream":
        return OracleStream(self, flags)

    def __del__(self):
        try:
            if self._h:
                lib().orc_model_free(self._h)
                self._h = None
        except Exception:
            pass


def _handles(streams):
    hs = (C.c_void_p * len(streams))(*[s._h for s in streams])
    return hs


def forward_batch(streams, audio, texts, want_logits: bool = True):
    """orc_forward for several streams of one model in one step (the same values each stream
    would get alone).  Returns (logits [n, vocab] or None, argmax [n])."""
    n = len(streams)
    a = np.ascontiguousarray(np.asarray(audio, dtype=np.uint32).reshape(n, -1))
    t = np.ascontiguousarray(np.asarray(texts, dtype=np.uint32).reshape(n))
    lg = np.empty((n, streams[0].model.vocab), dtype=np.float32) if want_logits else None
    am = np.empty(n, dtype=np.int64)
    rc = lib().orc_forward_batch(_handles(streams), n, _p(a, C.c_uint32), _p(t, C.c_uint32),
                                 _p(lg, C.c_float) if want_logits else None, _p(am, C.c_int64))
    if rc != 0:
        raise RuntimeError("oracle forward_batch failed: " + lib().orc_last_error().decode())
    return lg, am


def feed_frame_batch(streams, audio, want_logits: bool = False):
    """SttStream::feed_frame for several streams in one batched step.  Returns (tokens as a list
    with None for frames inside the delay, logits [n, vocab] or None)."""
    n = len(streams)
    a = np.ascontiguousarray(np.asarray(audio, dtype=np.uint32).reshape(n, -1))
    lg = np.empty((n, streams[0].model.vocab), dtype=np.float32) if want_logits else None
    tk = np.empty(n, dtype=np.int64)
    rc = lib().orc_feed_frame_batch(_handles(streams), n, _p(a, C.c_uint32), _p(lg, C.c_float) if want_logits else None,
                                    _p(tk, C.c_int64))
    if rc != 0:
        raise RuntimeError("oracle feed_frame_batch failed: " + lib().orc_last_error().decode())
    return [None if t < 0 else int(t) for t in tk], lg


class OracleStream:
    def __init__(self, model: OracleModel, flags: int = 0):
        self.model = model
        self._h = lib().orc_stream_new(model._h, flags)

    def forward(self, audio, text: int, want_logits: bool = True):
        a = np.ascontiguousarray(np.asarray(audio, dtype=np.uint32))
        lg = np.empty(self.model.vocab, dtype=np.float32) if want_logits else None
        r = lib().orc_forward(self._h, _p(a, C.c_uint32), text, _p(lg, C.c_float) if want_logits else None)
        if r < 0:
            raise RuntimeError("oracle forward failed: " + lib().orc_last_error().decode())
        return lg, int(r)

    def forward_gpu_token(self, audio, argmax, fallback_text: int):
        """SttModel::forward_with_gpu_token: `argmax` is the previous frame's argmax or None."""
        a = np.ascontiguousarray(np.asarray(audio, dtype=np.uint32))
        lg = np.empty(self.model.vocab, dtype=np.float32)
        r = lib().orc_forward_gpu_token(self._h, _p(a, C.c_uint32), 0 if argmax is None else 1,
                                        0 if argmax is None else int(argmax), fallback_text, _p(lg, C.c_float))
        if r < 0:
            raise RuntimeError("oracle forward_gpu_token failed: " + lib().orc_last_error().decode())
        return lg, int(r)

    def feed_frame_logits(self, audio):
        """feed_frame that also returns the step's logits: (token or None, logits)."""
        toks, lg = feed_frame_batch([self], np.asarray(audio).reshape(1, -1), want_logits=True)
        return toks[0], lg[0]

    def feed_frame(self, audio):
        a = np.ascontiguousarray(np.asarray(audio, dtype=np.uint32))
        r = lib().orc_feed_frame(self._h, _p(a, C.c_uint32))
        if r < -1:
            raise RuntimeError("oracle feed_frame failed: " + lib().orc_last_error().decode())
        return None if r == -1 else int(r)

    def flush(self):
        buf = np.zeros(64, dtype=np.uint32)
        n = lib().orc_flush(self._h, _p(buf, C.c_uint32), 64)
        if n < 0:
            raise RuntimeError("oracle flush failed: " + lib().orc_last_error().decode())
        return [int(x) for x in buf[:n]]

    def reset(self):
        lib().orc_stream_reset(self._h)

    def set_last_text_token(self, t: int):
        lib().orc_stream_set_last_text_token(self._h, t)

    def set_delay_state(self, last_text_token: int, prev0: int, prev1: int):
        lib().orc_stream_set_delay_state(self._h, last_text_token, prev0 & 0xFFFFFFFF, prev1 & 0xFFFFFFFF)

    def state(self) -> dict:
        out = (C.c_int64 * 7)()
        lib().orc_stream_state(self._h, out)
        k = ["offset", "len", "write_pos", "frame_count", "last_text_token", "prev0", "prev1"]
        return dict(zip(k, list(out)))

    def __del__(self):
        try:
            if self._h:
                lib().orc_stream_free(self._h)
                self._h = None
        except Exception:
            pass

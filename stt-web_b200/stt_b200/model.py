"""Host-side mirror of the stt-wasm model and stream API over the C ABI.

Names, argument meaning and error behaviour follow the reference crate:
  SttConfig           crates/stt-wasm/src/lib.rs:27-80
  SttModel            crates/stt-wasm/src/model.rs:583-752  (load = gguf.rs:752-826 + 658-692)
  LayerCaches         crates/stt-wasm/src/model.rs:262-296  (here: a set of N independent streams)
  SttStream           crates/stt-wasm/src/stream.rs:19-363
  Q4Tensor/q4_matmul  crates/stt-wasm/src/gguf.rs:403-578
Where the reference panics (bad token id, position past max_seq_len, shape mismatch), these
methods raise SttError.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, fields
from typing import List, Optional, Sequence

import numpy as np

from ._lib import (STT_KV_BF16, STT_KV_F32, SttError, check, lib, stt_config, stt_model_info,
                   stt_stream_state)


@dataclass
class SttConfig:
    """SttConfig (lib.rs:27-58); defaults are SttConfig::default() (lib.rs:60-80)."""
    num_layers: int = 16
    hidden_size: int = 2048
    num_heads: int = 16
    num_kv_heads: int = 16
    intermediate_size: int = 5632
    vocab_size: int = 8000
    text_in_vocab_size: int = 8001
    num_codebooks: int = 32
    audio_vocab_size: int = 2049
    text_delay: int = 6
    rope_theta: float = 100000.0
    max_seq_len: int = 4096
    sliding_window: int = 750
    text_padding_id: int = 3
    text_start_token: int = 8000

    def to_c(self) -> stt_config:
        c = stt_config()
        for f in fields(self):
            setattr(c, f.name, getattr(self, f.name))
        return c


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


def _ptr(a: np.ndarray, ct):
    return a.ctypes.data_as(C.POINTER(ct))


class SttModel:
    """The loaded STT transformer on one CUDA device."""

    def __init__(self, handle: C.c_void_p, config: SttConfig):
        self._h = handle
        self.config = config
        info = stt_model_info()
        check(lib().stt_model_get_info(self._h, C.byref(info)), "stt_model_get_info")
        self.info = info

    @classmethod
    def from_shards(cls, shards: Sequence[bytes | bytearray | memoryview | np.ndarray], device: int = 0,
                    config: Optional[SttConfig] = None) -> "SttModel":
        """Q4ModelLoader::from_shards + load_deferred + finalize (gguf.rs:752-826, 658-692)."""
        config = config or SttConfig()
        arrs = [np.frombuffer(s, dtype=np.uint8) if not isinstance(s, np.ndarray) else s.view(np.uint8)
                for s in shards]
        ptrs = (C.POINTER(C.c_uint8) * len(arrs))(*[_ptr(a, C.c_uint8) for a in arrs])
        lens = (C.c_size_t * len(arrs))(*[a.size for a in arrs])
        h = C.c_void_p()
        cfg = config.to_c()
        check(lib().stt_model_load_gguf(ptrs, lens, len(arrs), device, C.byref(cfg), C.byref(h)),
              "stt_model_load_gguf")
        return cls(h, config)

    @classmethod
    def from_buffer(cls, ptr: int, length: int, device: int = 0, config: Optional[SttConfig] = None) -> "SttModel":
        """Loads from one raw host buffer (address, length) without copying it into Python."""
        config = config or SttConfig()
        ptrs = (C.POINTER(C.c_uint8) * 1)(C.cast(C.c_void_p(ptr), C.POINTER(C.c_uint8)))
        lens = (C.c_size_t * 1)(length)
        h = C.c_void_p()
        cfg = config.to_c()
        check(lib().stt_model_load_gguf(ptrs, lens, 1, device, C.byref(cfg), C.byref(h)), "stt_model_load_gguf")
        return cls(h, config)

    def close(self) -> None:
        if self._h:
            lib().stt_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def create_cache(self, n_streams: int = 1, kv_dtype: str = "bf16") -> "LayerCaches":
        """SttModel::create_cache (model.rs:728-738) for n_streams independent streams."""
        return LayerCaches(self, n_streams, kv_dtype)

    def forward(self, audio_tokens, text_token: int, cache: "LayerCaches", stream_id: int = 0) -> np.ndarray:
        """SttModel::forward (model.rs:631-664): one step, returns logits [1, 1, vocab]."""
        logits, _ = cache.forward([stream_id], np.asarray(audio_tokens).reshape(1, -1), [text_token])
        return logits.reshape(1, 1, -1)


class LayerCaches:
    """N independent streams: per-layer K/V rings of sliding_window+1 slots plus step state."""

    def __init__(self, model: SttModel, n_streams: int, kv_dtype: str = "bf16"):
        self.model = model
        self.n_streams = n_streams
        kv = {"bf16": STT_KV_BF16, "f32": STT_KV_F32}[kv_dtype]
        h = C.c_void_p()
        check(lib().stt_streams_create(model._h, n_streams, kv, C.byref(h)), "stt_streams_create")
        self._h = h

    def close(self) -> None:
        if self._h:
            lib().stt_streams_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, stream_ids: Sequence[int], audio: np.ndarray, text: Sequence[int],
                want_logits: bool = True):
        """Batched raw step: returns (logits [n, vocab] or None, argmax [n])."""
        ids = np.ascontiguousarray(np.asarray(stream_ids, dtype=np.int32))
        n = ids.size
        a = _u32(audio).reshape(n, -1)
        t = _u32(text).reshape(n)
        V = self.model.info.vocab_size
        logits = np.empty((n, V), dtype=np.float32) if want_logits else None
        am = np.empty(n, dtype=np.uint32)
        check(lib().stt_forward(self._h, _ptr(ids, C.c_int32), n, _ptr(a, C.c_uint32), _ptr(t, C.c_uint32),
                                _ptr(logits, C.c_float) if want_logits else None, _ptr(am, C.c_uint32)),
              "stt_forward")
        return logits, am

    def feed_frame(self, stream_ids: Sequence[int], audio: np.ndarray) -> np.ndarray:
        """One batched feed_frame step; returns emitted tokens (-1 = None)."""
        ids = np.ascontiguousarray(np.asarray(stream_ids, dtype=np.int32))
        a = _u32(audio).reshape(ids.size, -1)
        out = np.empty(ids.size, dtype=np.int32)
        check(lib().stt_streams_feed_frame(self._h, _ptr(ids, C.c_int32), ids.size, _ptr(a, C.c_uint32),
                                           _ptr(out, C.c_int32)), "stt_streams_feed_frame")
        return out

    def submit_frame(self, stream_ids: Sequence[int], audio: np.ndarray) -> "PendingFrame":
        """Queues one batched feed_frame step without waiting (SttStream::submit_frame_gpu,
        stream.rs:117-138); its tokens are taken later from the returned PendingFrame."""
        ids = np.ascontiguousarray(np.asarray(stream_ids, dtype=np.int32))
        a = _u32(audio).reshape(ids.size, -1)
        t = C.c_int64()
        check(lib().stt_streams_submit_frame(self._h, _ptr(ids, C.c_int32), ids.size, _ptr(a, C.c_uint32),
                                             C.byref(t)), "stt_streams_submit_frame")
        return PendingFrame(self, t.value, ids.size)

    def state(self, stream_id: int) -> dict:
        st = stt_stream_state()
        check(lib().stt_stream_get_state(self._h, stream_id, C.byref(st)), "stt_stream_get_state")
        return {"offset": st.offset, "len": st.len, "write_pos": st.write_pos, "frame_count": st.frame_count,
                "last_text_token": st.last_text_token, "delay_prev": (st.delay_prev[0], st.delay_prev[1])}

    def reset(self, stream_id: int = 0, keep_buffers: bool = False) -> None:
        check(lib().stt_stream_reset(self._h, stream_id, 1 if keep_buffers else 0), "stt_stream_reset")


class PendingFrame:
    """A submitted batched frame (the analogue of a PendingFrame of take_batch_pending,
    stream.rs:146-183): poll() returns its tokens once its step has completed (None before),
    wait() blocks for them.  Tokens are -1 where a stream is still inside the text delay."""

    def __init__(self, cache: "LayerCaches", ticket: int, n: int):
        self.cache, self.ticket, self.n = cache, ticket, n

    def poll(self) -> Optional[np.ndarray]:
        out = np.empty(self.n, dtype=np.int32)
        ready = C.c_int()
        check(lib().stt_streams_poll_frame(self.cache._h, self.ticket, _ptr(out, C.c_int32), C.byref(ready)),
              "stt_streams_poll_frame")
        return out if ready.value else None

    def wait(self) -> np.ndarray:
        out = np.empty(self.n, dtype=np.int32)
        check(lib().stt_streams_wait_frame(self.cache._h, self.ticket, _ptr(out, C.c_int32)), "stt_streams_wait_frame")
        return out


class SttStream:
    """SttStream (stream.rs:19-363) bound to one stream of a LayerCaches set."""

    def __init__(self, config: SttConfig, cache: LayerCaches, stream_id: int = 0):
        self.config = config
        self.cache = cache
        self.stream_id = stream_id

    def _check_model(self, model: Optional[SttModel]) -> None:
        if model is not None and model is not self.cache.model:
            raise SttError(-1, "SttStream: the model differs from the one the cache was created for")

    def feed_frame(self, audio_tokens, model: Optional[SttModel] = None) -> Optional[int]:
        """stream.rs:70-81: returns the emitted token or None during the text delay."""
        self._check_model(model)
        a = _u32(audio_tokens)
        tok = C.c_int32()
        check(lib().stt_stream_feed_frame(self.cache._h, self.stream_id, _ptr(a, C.c_uint32), C.byref(tok)),
              "stt_stream_feed_frame")
        return None if tok.value < 0 else int(tok.value)

    def feed_frames(self, audio_frames, model: Optional[SttModel] = None) -> List[Optional[int]]:
        """Many feed_frame calls, run back to back on the device."""
        self._check_model(model)
        a = _u32(audio_frames)
        n = a.size // self.config.num_codebooks
        out = np.empty(n, dtype=np.int32)
        check(lib().stt_stream_feed_frames(self.cache._h, self.stream_id, n, _ptr(a, C.c_uint32),
                                           _ptr(out, C.c_int32)), "stt_stream_feed_frames")
        return [None if t < 0 else int(t) for t in out]

    def flush(self, model: Optional[SttModel] = None) -> List[int]:
        """stream.rs:315-338: text_delay zero-audio frames, emitted tokens collected."""
        self._check_model(model)
        cap = max(1, self.config.text_delay)
        buf = np.zeros(cap, dtype=np.uint32)
        n = C.c_int()
        check(lib().stt_stream_flush(self.cache._h, self.stream_id, _ptr(buf, C.c_uint32), cap, C.byref(n)),
              "stt_stream_flush")
        return [int(x) for x in buf[:n.value]]

    def reset(self) -> None:
        """stream.rs:341-349."""
        self.cache.reset(self.stream_id, keep_buffers=False)

    def reset_keep_buffers(self) -> None:
        """stream.rs:354-362."""
        self.cache.reset(self.stream_id, keep_buffers=True)

    def set_last_text_token(self, token: int) -> None:
        """stream.rs:190-192."""
        check(lib().stt_stream_set_last_text_token(self.cache._h, self.stream_id, token),
              "stt_stream_set_last_text_token")

    @property
    def frame_count(self) -> int:
        return self.cache.state(self.stream_id)["frame_count"]


class Q4Tensor:
    """Q4Tensor (gguf.rs:403-460): one Q4_0 matrix [n, k] in the device layout."""

    def __init__(self, handle, shape, device):
        self._h = handle
        self.shape = shape
        self.device = device

    @classmethod
    def from_q4_bytes(cls, raw: bytes | np.ndarray, shape, device: int = 0) -> "Q4Tensor":
        n, k = shape
        a = np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray) else np.ascontiguousarray(raw, np.uint8)
        h = C.c_void_p()
        check(lib().stt_q4_tensor_create(_ptr(a, C.c_uint8), a.size, n, k, device, C.byref(h)),
              "stt_q4_tensor_create")
        return cls(h, (n, k), device)

    def close(self):
        if self._h:
            lib().stt_q4_tensor_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def status(self) -> None:
        """Waits for the device; raises SttError (STT_E_DEVICE_FLAG) if a device-side wait of a
        matmul on this tensor ran out since the last check (that output is invalid)."""
        check(lib().stt_q4_tensor_status(self._h), "stt_q4_tensor_status")

    def dequant(self) -> np.ndarray:
        out = np.empty(self.shape, dtype=np.float32)
        check(lib().stt_q4_tensor_dequant(self._h, _ptr(out, C.c_float)), "stt_q4_tensor_dequant")
        return out


def q4_matmul(inp: np.ndarray, weights: Q4Tensor) -> np.ndarray:
    """q4_matmul (gguf.rs:517-578): output[B, M, N] = input[B, M, K] x weights[N, K]^T."""
    x = np.ascontiguousarray(np.asarray(inp, dtype=np.float32))
    if x.ndim != 3:
        raise SttError(-1, "q4_matmul: input must be 3-D [B, M, K]")
    B, M, K = x.shape
    n, k = weights.shape
    if K != k:
        raise SttError(-1, f"q4_matmul: K dimension mismatch: input has {K}, weights have {k}")
    out = np.empty((B, M, n), dtype=np.float32)
    check(lib().stt_q4_matmul(weights._h, _ptr(x, C.c_float), B * M, _ptr(out, C.c_float)), "stt_q4_matmul")
    return out

"""SentencePiece detokeniser with the API of the reference's SpmDecoder
(crates/stt-wasm/src/tokenizer.rs:7-38): token ids emitted by a stream become text.

Thin wrapper over stt_spm_* in libsttb200 (csrc/spm.cpp); host only, no device needed.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import check, lib


class SpmDecoder:
    """Maps token ids to text with the reference's rules: ids 0 and 3 skipped, byte-fallback runs
    kept only when they are valid UTF-8, U+2581 as a space, no trimming (tokenizer.rs:150-192)."""

    def __init__(self, handle):
        self._h = handle

    @classmethod
    def from_bytes(cls, data) -> "SpmDecoder":
        """SpmDecoder::from_bytes (tokenizer.rs:14-17): parses a SentencePiece `.model` protobuf."""
        buf = np.frombuffer(bytes(data), dtype=np.uint8)
        h = C.c_void_p()
        check(lib().stt_spm_decoder_create(buf.ctypes.data_as(C.POINTER(C.c_uint8)), buf.size, C.byref(h)),
              "stt_spm_decoder_create")
        return cls(h)

    @classmethod
    def load(cls, path: str) -> "SpmDecoder":
        """SpmDecoder::load on a native host (tokenizer.rs:23-26, 217-220): reads the file."""
        with open(path, "rb") as f:
            return cls.from_bytes(f.read())

    def vocab_len(self) -> int:
        n = C.c_int64()
        check(lib().stt_spm_vocab_len(self._h, C.byref(n)), "stt_spm_vocab_len")
        return n.value

    @staticmethod
    def _text(call, where) -> str:
        n = C.c_size_t()
        check(call(None, 0, C.byref(n)), where)
        buf = C.create_string_buffer(n.value + 1)
        check(call(buf, n.value + 1, C.byref(n)), where)
        return buf.raw[:n.value].decode("utf-8")

    def piece(self, token_id: int) -> str:
        return self._text(lambda o, c, n: lib().stt_spm_piece(self._h, token_id, o, c, n), "stt_spm_piece")

    def decode(self, ids) -> str:
        """SpmDecoder::decode (tokenizer.rs:30-32)."""
        a = np.ascontiguousarray(np.asarray(list(ids) if not isinstance(ids, np.ndarray) else ids, dtype=np.uint32))
        p = a.ctypes.data_as(C.POINTER(C.c_uint32))
        return self._text(lambda o, c, n: lib().stt_spm_decode(self._h, p, a.size, o, c, n), "stt_spm_decode")

    def close(self):
        if self._h:
            lib().stt_spm_decoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

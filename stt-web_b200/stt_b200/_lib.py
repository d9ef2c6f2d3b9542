"""ctypes bindings of libsttb200 (include/stt_b200.h).

The shared library is built in-tree next to this file (``make -C stt-web_b200``).  Loading fails
loudly when it is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsttb200.so")

STT_OK = 0
STT_E_INVALID_ARG = -1
STT_E_FORMAT = -2
STT_E_OOM = -3
STT_E_CUDA = -4
STT_E_DEVICE_FLAG = -5
STT_E_STATE = -6

STT_KV_BF16 = 0
STT_KV_F32 = 1

STT_PRODUCTS_F16X3 = 0
STT_PRODUCTS_F16X2 = 1

GGML_F32, GGML_F16, GGML_Q4_0, GGML_BF16 = 0, 1, 2, 30


class stt_config(C.Structure):
    _fields_ = [
        ("num_layers", C.c_int32),
        ("hidden_size", C.c_int32),
        ("num_heads", C.c_int32),
        ("num_kv_heads", C.c_int32),
        ("intermediate_size", C.c_int32),
        ("vocab_size", C.c_int32),
        ("text_in_vocab_size", C.c_int32),
        ("num_codebooks", C.c_int32),
        ("audio_vocab_size", C.c_int32),
        ("text_delay", C.c_int32),
        ("rope_theta", C.c_double),
        ("max_seq_len", C.c_int32),
        ("sliding_window", C.c_int32),
        ("text_padding_id", C.c_uint32),
        ("text_start_token", C.c_uint32),
    ]


class stt_model_info(C.Structure):
    _fields_ = [
        ("num_layers", C.c_int32),
        ("hidden_size", C.c_int32),
        ("num_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("ffn_hidden", C.c_int32),
        ("vocab_size", C.c_int32),
        ("text_in_vocab_size", C.c_int32),
        ("num_codebooks", C.c_int32),
        ("audio_vocab_size", C.c_int32),
        ("embedding_dtype", C.c_int32),
        ("device", C.c_int32),
        ("q4_weight_bytes", C.c_uint64),
        ("device_bytes", C.c_uint64),
        ("tensor_core_min_batch", C.c_int32),
        ("reserved", C.c_int32),
    ]


class stt_stream_state(C.Structure):
    _fields_ = [
        ("offset", C.c_int32),
        ("len", C.c_int32),
        ("write_pos", C.c_int32),
        ("frame_count", C.c_int32),
        ("last_text_token", C.c_uint32),
        ("delay_prev", C.c_uint32 * 2),
    ]


P = C.c_void_p
U8P = C.POINTER(C.c_uint8)
U32P = C.POINTER(C.c_uint32)
I32P = C.POINTER(C.c_int32)
F32P = C.POINTER(C.c_float)

# name -> (restype, argtypes); every symbol declared in include/stt_b200.h
SIGNATURES = {
    "stt_config_default": (None, [C.POINTER(stt_config)]),
    "stt_model_load_gguf": (C.c_int, [C.POINTER(U8P), C.POINTER(C.c_size_t), C.c_int, C.c_int,
                                      C.POINTER(stt_config), C.POINTER(P)]),
    "stt_model_destroy": (C.c_int, [P]),
    "stt_model_get_info": (C.c_int, [P, C.POINTER(stt_model_info)]),
    "stt_streams_create": (C.c_int, [P, C.c_int, C.c_int, C.POINTER(P)]),
    "stt_streams_destroy": (C.c_int, [P]),
    "stt_forward": (C.c_int, [P, I32P, C.c_int, U32P, U32P, F32P, U32P]),
    "stt_stream_feed_frame": (C.c_int, [P, C.c_int, U32P, I32P]),
    "stt_streams_feed_frame": (C.c_int, [P, I32P, C.c_int, U32P, I32P]),
    "stt_stream_feed_frames": (C.c_int, [P, C.c_int, C.c_int, U32P, I32P]),
    "stt_stream_feed_frames_device": (C.c_int, [P, C.c_int, C.c_int, P, P, P]),
    "stt_streams_feed_frame_device": (C.c_int, [P, I32P, C.c_int, P, P, P]),
    "stt_streams_submit_frame": (C.c_int, [P, I32P, C.c_int, U32P, C.POINTER(C.c_int64)]),
    "stt_streams_poll_frame": (C.c_int, [P, C.c_int64, I32P, C.POINTER(C.c_int)]),
    "stt_streams_wait_frame": (C.c_int, [P, C.c_int64, I32P]),
    "stt_stream_flush": (C.c_int, [P, C.c_int, U32P, C.c_int, I32P]),
    "stt_stream_reset": (C.c_int, [P, C.c_int, C.c_int]),
    "stt_stream_reset_async": (C.c_int, [P, C.c_int, C.c_int, P]),
    "stt_stream_set_last_text_token": (C.c_int, [P, C.c_int, C.c_uint32]),
    "stt_streams_set_product_precision": (C.c_int, [P, C.c_int]),
    "stt_stream_get_state": (C.c_int, [P, C.c_int, C.POINTER(stt_stream_state)]),
    "stt_q4_tensor_create": (C.c_int, [U8P, C.c_size_t, C.c_int, C.c_int, C.c_int, C.POINTER(P)]),
    "stt_q4_tensor_destroy": (C.c_int, [P]),
    "stt_q4_matmul": (C.c_int, [P, F32P, C.c_int, F32P]),
    "stt_q4_matmul_device": (C.c_int, [P, P, C.c_int, C.c_int, P, P]),
    "stt_q4_tensor_dequant": (C.c_int, [P, F32P]),
    "stt_q4_tensor_status": (C.c_int, [P]),
    "stt_q4_matmul_device_noalloc": (C.c_int, [P, P, C.c_int, C.c_int, C.c_int, P, P]),
    "stt_spm_decoder_create": (C.c_int, [U8P, C.c_size_t, C.POINTER(P)]),
    "stt_spm_decoder_destroy": (C.c_int, [P]),
    "stt_spm_vocab_len": (C.c_int, [P, C.POINTER(C.c_int64)]),
    "stt_spm_piece": (C.c_int, [P, C.c_int64, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "stt_spm_decode": (C.c_int, [P, U32P, C.c_size_t, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "stt_debug_trace_frame": (C.c_int, [P, C.c_int]),
    "stt_debug_get_trace": (C.c_int, [P, C.POINTER(C.c_uint64), C.c_int, I32P]),
    "stt_debug_get_trace_ctas": (C.c_int, [P, C.POINTER(C.c_uint64), C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "stt_debug_barrier_ns": (C.c_int, [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double)]),
    "stt_debug_graph_kernels": (C.c_int, [P, C.c_int, C.POINTER(C.c_int)]),
    "stt_debug_arm_wait_timeout": (C.c_int, [P]),
    "stt_debug_q4_arm_wait_timeout": (C.c_int, [P]),
    "stt_debug_fail_allocation": (C.c_int, [C.c_int]),
    "stt_debug_time_products": (C.c_int, [P, C.c_int, C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "stt_last_error": (C.c_char_p, []),
}

_lib = None


def lib() -> C.CDLL:
    """Loads libsttb200.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `make -C stt-web_b200` (there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


class SttError(RuntimeError):
    """An STT_E_* status returned by the library."""

    def __init__(self, code: int, where: str):
        msg = lib().stt_last_error().decode("utf-8", "replace")
        super().__init__(f"{where}: status {code}: {msg}")
        self.code = code


def check(code: int, where: str) -> None:
    if code != STT_OK:
        raise SttError(code, where)

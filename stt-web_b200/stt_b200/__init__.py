"""stt_b200 — B200-native (sm_100a) STT-1B decode step with the stt-wasm model/stream API.

Add the directory holding this package (``stt-web_b200``) to ``sys.path`` and import
``stt_b200``.  The CUDA library ``libsttb200.so`` must be built first (``make -C stt-web_b200``).
"""
from ._lib import LIB_PATH, SttError, lib  # noqa: F401
from .model import LayerCaches, PendingFrame, Q4Tensor, SttConfig, SttModel, SttStream, q4_matmul  # noqa: F401
from .synth import SynthSpec, audio_tokens, quantize_q4_0, synth_gguf  # noqa: F401
from .tokenizer import SpmDecoder  # noqa: F401

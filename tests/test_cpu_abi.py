"""The C ABI without a GPU: exported symbols, defaults, and the loader's validation of GGUF bytes
(which the library completes before it touches a device)."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import REPO, has_gpu
from gguf_tools import split_tensors, write_gguf
import stt_b200
from stt_b200 import _lib
from stt_b200.model import SttConfig


def header_functions(header="stt_b200.h"):
    text = open(os.path.join(REPO, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(stt_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = header_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(L, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_generator_library_is_separate_from_the_decode_library():
    """The synthetic-checkpoint generator lives in its own host-only library: the decode library
    neither exports it nor needs it, and the generator library has no CUDA dependency."""
    from stt_b200 import synth
    S = synth.synth_lib()
    names = header_functions("stt_synth.h")
    assert len(names) == 6
    for n in names:
        assert hasattr(S, n), n
        assert n in synth.SYNTH_SIGNATURES, f"{n} has no ctypes signature"
        assert not hasattr(_lib.lib(), n), f"{n} is exported by the decode library"
    needed = subprocess.run(["readelf", "-d", synth.SYNTH_LIB_PATH], capture_output=True, text=True).stdout
    assert "cuda" not in needed.lower()


def test_oracle_is_not_linked_into_the_library():
    data = open(_lib.LIB_PATH, "rb").read()
    assert b"orc_" not in data


def test_config_defaults_match_reference():
    c = _lib.stt_config()
    _lib.lib().stt_config_default(C.byref(c))
    # SttConfig::default, crates/stt-wasm/src/lib.rs:60-80
    ref = dict(num_layers=16, hidden_size=2048, num_heads=16, num_kv_heads=16, intermediate_size=5632,
               vocab_size=8000, text_in_vocab_size=8001, num_codebooks=32, audio_vocab_size=2049, text_delay=6,
               rope_theta=100000.0, max_seq_len=4096, sliding_window=750, text_padding_id=3, text_start_token=8000)
    for k, v in ref.items():
        assert getattr(c, k) == v, k
        assert getattr(SttConfig(), k) == v, k


def load_status(buf: bytes, cfg: SttConfig | None = None, shards=None):
    a = np.frombuffer(buf, np.uint8)
    parts = shards or [a]
    ptrs = (C.POINTER(C.c_uint8) * len(parts))(*[p.ctypes.data_as(C.POINTER(C.c_uint8)) for p in parts])
    lens = (C.c_size_t * len(parts))(*[p.size for p in parts])
    h = C.c_void_p()
    cc = (cfg or tiny_cfg()).to_c()
    rc = _lib.lib().stt_model_load_gguf(ptrs, lens, len(parts), 0, C.byref(cc), C.byref(h))
    msg = _lib.lib().stt_last_error().decode()
    if rc == 0:
        _lib.lib().stt_model_destroy(h)
    return rc, msg


def tiny_cfg():
    return SttConfig(num_layers=2, hidden_size=256, num_heads=2, num_kv_heads=2, num_codebooks=4,
                     text_start_token=1000, vocab_size=1000, text_in_vocab_size=1001, audio_vocab_size=300)


def valid_status():
    return 0 if has_gpu() else _lib.STT_E_CUDA


def test_reference_written_file_passes_validation(tiny_ref_gguf):
    rc, msg = load_status(tiny_ref_gguf.tobytes())
    assert rc == valid_status(), msg


def test_sharded_input_passes_validation(tiny_ref_gguf):
    a = tiny_ref_gguf
    cuts = [0, 7, 1001, 500_003, a.size]
    shards = [np.ascontiguousarray(a[cuts[i]:cuts[i + 1]]) for i in range(len(cuts) - 1)]
    rc, msg = load_status(b"", shards=shards)
    assert rc == valid_status(), msg


def mutate(tiny_ref_gguf, fn):
    ts = split_tensors(tiny_ref_gguf.tobytes())
    ts = fn(ts)
    return write_gguf(ts, {"general.architecture": "kyutai-stt"})


@pytest.mark.parametrize("case,pattern", [
    ("magic", "Invalid GGUF magic"),
    ("version", "Unsupported GGUF version: 4"),
    ("meta_type", "Unknown GGUF metadata value type: 13"),
    ("dtype", "Unsupported GGML dtype code: 7"),
    ("truncated", "runs past the end"),
    ("header_cut", "Failed to read"),
    ("missing", "Tensor 'transformer.layers.1.gating.linear_out.weight' not found"),
    ("linear_f32", "Expected Q4_0 for 'text_linear.weight'"),
    ("norm_q4", "Cannot load Q4_0 tensor 'out_norm.alpha' as norm weight"),
    ("bad_utf8", "Invalid UTF-8"),
    ("shape", "has shape"),
])
def test_loader_rejects_malformed_files(tiny_ref_gguf, case, pattern):
    if case == "magic":
        buf = bytearray(tiny_ref_gguf.tobytes())
        buf[0] = ord("X")
    elif case == "version":
        buf = bytearray(tiny_ref_gguf.tobytes())
        buf[4:8] = (4).to_bytes(4, "little")
    elif case == "meta_type":
        buf = write_gguf(split_tensors(tiny_ref_gguf.tobytes()), {"x": ("raw", 13, b"")})
    elif case == "dtype":
        def f(ts):
            name, shape, dt, data = ts[0]
            return [(name, shape, 7, data)] + ts[1:]
        buf = mutate(tiny_ref_gguf, f)
    elif case == "truncated":
        buf = tiny_ref_gguf.tobytes()[:-100]
    elif case == "header_cut":
        buf = tiny_ref_gguf.tobytes()[:40]
    elif case == "missing":
        buf = mutate(tiny_ref_gguf, lambda ts: [t for t in ts if t[0] != "transformer.layers.1.gating.linear_out.weight"])
    elif case == "linear_f32":
        def f(ts):
            out = []
            for name, shape, dt, data in ts:
                if name == "text_linear.weight":
                    data = np.zeros(int(np.prod(shape)), np.float32).tobytes()
                    dt = 0
                out.append((name, shape, dt, data))
            return out
        buf = mutate(tiny_ref_gguf, f)
    elif case == "norm_q4":
        def f(ts):
            out = []
            for name, shape, dt, data in ts:
                if name == "out_norm.alpha":
                    data = bytes(int(np.prod(shape)) // 32 * 18)
                    dt = 2
                out.append((name, shape, dt, data))
            return out
        buf = mutate(tiny_ref_gguf, f)
    elif case == "bad_utf8":
        def f(ts):
            name, shape, dt, data = ts[0]
            return [("\udcff" + name, shape, dt, data)] + ts[1:]
        ts = split_tensors(tiny_ref_gguf.tobytes())
        good = write_gguf(ts, {})
        # overwrite the first byte of the first tensor name with an invalid UTF-8 byte
        i = good.index(ts[0][0].encode())
        b = bytearray(good)
        b[i] = 0xFF
        buf = bytes(b)
    elif case == "shape":
        def f(ts):
            out = []
            for name, shape, dt, data in ts:
                if name == "transformer.layers.0.self_attn.out_proj.weight":
                    shape = (shape[0] // 2, shape[1] * 2)
                out.append((name, shape, dt, data))
            return out
        buf = mutate(tiny_ref_gguf, f)
    rc, msg = load_status(bytes(buf))
    assert rc == _lib.STT_E_FORMAT, (rc, msg)
    assert pattern in msg, msg


def test_bad_config_is_rejected(tiny_ref_gguf):
    cfg = tiny_cfg()
    cfg.num_kv_heads = 1
    rc, msg = load_status(tiny_ref_gguf.tobytes(), cfg)
    assert rc == _lib.STT_E_INVALID_ARG and "MHA" in msg


def test_errors_do_not_need_a_device():
    with pytest.raises(stt_b200.SttError) as e:
        stt_b200.SttModel.from_shards([b"nope"], config=tiny_cfg())
    assert e.value.code == _lib.STT_E_FORMAT

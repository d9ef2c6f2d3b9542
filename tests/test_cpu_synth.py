"""The synthetic checkpoint generator: quantize.py-exact Q4_0, the reference's file layout,
determinism, and the audio-token source."""
import os

import numpy as np

from conftest import GOLDEN
from gguf_tools import read_gguf, split_tensors
import stt_b200
from oracle import oracle as O

SMALL = dict(num_layers=2, hidden_size=256, num_heads=2, ffn_hidden=512, vocab_size=1000, text_in_vocab_size=1001,
             num_codebooks=4, audio_vocab_size=300)


def test_generator_quantizer_matches_quantize_py():
    z = np.load(os.path.join(GOLDEN, "q4_quantize.npz"))
    with np.errstate(all="ignore"):
        got = stt_b200.quantize_q4_0(z["x"])
    assert np.array_equal(got, z["q"])


def test_generator_is_deterministic_and_seeded():
    a = stt_b200.synth_gguf(stt_b200.SynthSpec(seed=1, **SMALL)).array.copy()
    b = stt_b200.synth_gguf(stt_b200.SynthSpec(seed=1, n_threads=3, **SMALL)).array.copy()
    c = stt_b200.synth_gguf(stt_b200.SynthSpec(seed=2, **SMALL)).array.copy()
    assert np.array_equal(a, b)
    assert a.size == c.size and not np.array_equal(a, c)


def test_generator_file_layout_follows_quantize_py():
    for edt in (30, 2, 0):
        g = stt_b200.synth_gguf(stt_b200.SynthSpec(seed=3, embedding_dtype=edt, **SMALL))
        buf = g.array.tobytes()
        version, ts, data_off = read_gguf(buf)
        assert version == 3 and data_off % 32 == 0
        names = sorted(ts, key=lambda n: ts[n]["order"])
        assert names == sorted(names)                      # sorted-name order (quantize.py:268)
        offs = [ts[n]["offset"] for n in names]
        assert offs[0] == 0 and offs == sorted(offs)       # packed back to back
        D, F = SMALL["hidden_size"], SMALL["ffn_hidden"]
        assert ts["text_linear.weight"]["dims"] == [D, SMALL["vocab_size"]]  # GGUF dims are reversed
        assert ts["transformer.layers.1.gating.linear_in.weight"]["dims"] == [D, 2 * F]
        assert ts["transformer.layers.1.gating.linear_out.weight"]["dims"] == [F, D]
        assert ts["out_norm.alpha"]["dims"] == [D, 1, 1] and ts["out_norm.alpha"]["dtype"] == 0
        assert ts["emb.3.weight"]["dtype"] == edt and ts["text_emb.weight"]["dtype"] == edt
        assert ts["transformer.layers.0.self_attn.in_proj_weight"]["dtype"] == 2
        assert len(buf) == data_off + offs[-1] + {0: 4, 1: 2, 2: 18 / 32, 30: 2}[ts[names[-1]]["dtype"]] * int(
            np.prod(ts[names[-1]]["dims"]))


def test_generated_values_have_the_requested_distribution():
    g = stt_b200.synth_gguf(stt_b200.SynthSpec(seed=4, **SMALL))
    t = {n: (s, d, b) for n, s, d, b in split_tensors(g.array.tobytes())}
    s, d, b = t["transformer.layers.0.gating.linear_in.weight"]
    w = O.dequant_q4_0(np.frombuffer(b, np.uint8), s[0], s[1])
    assert abs(w.std() - 0.02) < 0.002 and abs(w.mean()) < 1e-3
    s, d, b = t["emb.0.weight"]
    e = (np.frombuffer(b, np.uint16).astype(np.uint32) << 16).view(np.float32)
    assert abs(e.std() - 0.02) < 0.001
    s, d, b = t["out_norm.alpha"]
    a = np.frombuffer(b, np.float32)
    assert abs(a.mean() - 1.0) < 0.01 and abs(a.std() - 0.02) < 0.005
    # norm alphas and embeddings are bf16 values
    assert np.all((a.view(np.uint32) & 0xFFFF) == 0)


def test_oracle_runs_on_generated_checkpoint():
    for edt in (30, 2):
        g = stt_b200.synth_gguf(stt_b200.SynthSpec(seed=5, embedding_dtype=edt, **SMALL))
        m = O.OracleModel(g.array, num_layers=2, num_heads=2, num_codebooks=4, text_start_token=1000)
        s = m.stream()
        lg, am = s.forward(np.arange(4, dtype=np.uint32), 1000)
        assert np.isfinite(lg).all() and 0 <= am < 1000 and 0.3 < lg.std() < 3


def test_audio_tokens():
    a = stt_b200.audio_tokens(7, 0, 50)
    assert a.shape == (50, 32) and a.max() < 2048 and a.min() >= 0
    assert np.array_equal(a, stt_b200.audio_tokens(7, 0, 50))
    assert not np.array_equal(a, stt_b200.audio_tokens(7, 1, 50))
    assert np.array_equal(a[10:], stt_b200.audio_tokens(7, 0, 40, first_frame=10))
    counts = np.bincount(stt_b200.audio_tokens(1, 3, 2000).ravel(), minlength=2048)
    assert counts.min() > 5 and counts.max() < 70

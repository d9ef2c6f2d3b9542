"""Pins the CPU oracle to the reference: golden vectors from scripts/quantize.py and the restated
cases of crates/stt-wasm/tests/q4_matmul.rs, plus an independent float64 restatement of model.rs."""
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import oracle as O
from gguf_tools import split_tensors


def test_f16_gguf_conversion_matches_reference_rule():
    golden = np.load(os.path.join(GOLDEN, "f16_gguf.npy"))
    got = np.array([np.float32(O.f16_to_f32_gguf(b)).view(np.uint32) for b in range(65536)], dtype=np.uint32)
    # NaN payloads survive the ctypes float round trip as NaN; compare those by class
    nan = (golden & 0x7F800000) == 0x7F800000
    nan &= (golden & 0x7FFFFF) != 0
    assert np.array_equal(got[~nan], golden[~nan])
    assert np.isnan(got[nan].view(np.float32)).all()


def test_f16_ieee_conversion_matches_numpy():
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([O.f16_to_f32_ieee(int(b)) for b in bits], dtype=np.float32)
    ok = ~np.isnan(ref)
    assert np.array_equal(got[ok].view(np.uint32), ref[ok].view(np.uint32))
    # the two conversions differ exactly on the subnormals, where gguf.rs gives half the value
    g = np.load(os.path.join(GOLDEN, "f16_gguf.npy")).view(np.float32)
    sub = (bits & 0x7C00) == 0
    sub &= (bits & 0x3FF) != 0
    assert np.array_equal(g[sub] * 2, ref[sub])
    assert np.array_equal(g[~sub & ok].view(np.uint32), ref[~sub & ok].view(np.uint32))


def test_quantizer_matches_quantize_py():
    z = np.load(os.path.join(GOLDEN, "q4_quantize.npz"))
    with np.errstate(all="ignore"):
        got = O.quantize_q4_0(z["x"])
    assert np.array_equal(got, z["q"])


def test_dequant_rule():
    z = np.load(os.path.join(GOLDEN, "q4_quantize.npz"))
    raw = z["q"][: 18 * 64]
    deq = O.dequant_q4_0(raw, 1, 64 * 32)[0]
    blocks = raw.reshape(-1, 18)
    scale = blocks[:, :2].copy().view(np.float16).astype(np.float32).ravel()
    lo = (blocks[:, 2:] & 0x0F).astype(np.float32) - 8
    hi = (blocks[:, 2:] >> 4).astype(np.float32) - 8
    ref = (np.concatenate([lo, hi], axis=1) * scale[:, None]).ravel()
    assert np.array_equal(deq, ref.astype(np.float32))


@pytest.mark.parametrize("case", ["identity", "different_inputs", "larger_realistic", "embedding_sum"])
def test_q4_matmul_reference_cases(case):
    z = np.load(os.path.join(GOLDEN, "q4_matmul_kats.npz"))
    n, k = z[f"{case}__shape"]
    x = z[f"{case}__x"]
    out = O.q4_matmul(z[f"{case}__raw"], int(n), int(k), x)
    exp = z[f"{case}__expected"]
    tol = float(z[f"{case}__tol"][0])
    if tol > 0:  # the reference test's own bound (q4_matmul.rs:151, 228, 306)
        assert np.abs(out - exp).max() < tol
    # and far tighter: both are f32 sums of the same exact products
    assert np.abs(out - exp).max() <= 1e-5 * max(1.0, np.abs(exp).max())
    # distinct inputs give distinct outputs (q4_matmul.rs:196-210, 275-289, 374-388)
    for i in range(len(x)):
        for j in range(i + 1, len(x)):
            assert np.abs(out[i] - out[j]).sum() > 1.0


def test_q4_matmul_vs_float64():
    rng = np.random.default_rng(3)
    n, k = 96, 512
    raw = O.quantize_q4_0((rng.standard_normal(n * k) * 0.02).astype(np.float32))
    x = rng.standard_normal((3, k)).astype(np.float32)
    w = O.dequant_q4_0(raw, n, k).astype(np.float64)
    ref = x.astype(np.float64) @ w.T
    got = O.q4_matmul(raw, n, k, x)
    assert np.abs(got - ref).max() < 1e-5 * np.abs(ref).max()


# ---------------------------------------------------------------- independent float64 model


class F64Model:
    """model.rs restated in float64 numpy, for the tiny checkpoint written by quantize.py."""

    def __init__(self, buf, meta):
        self.meta = meta
        t = {name: (shape, dtype, data) for name, shape, dtype, data in split_tensors(buf.tobytes())}
        D = meta["hidden"]

        def q4(name):
            shape, dtype, data = t[name]
            assert dtype == 2
            return O.dequant_q4_0(np.frombuffer(data, np.uint8), shape[0], shape[1]).astype(np.float64)

        def norm(name):
            shape, dtype, data = t[name]
            return np.frombuffer(data, np.float32).astype(np.float64)

        def emb(name):
            shape, dtype, data = t[name]
            raw = np.frombuffer(data, np.uint8).reshape(shape[0], -1)
            # gguf.rs dequant (scales are normal here, so IEEE == gguf.rs conversion)
            return O.dequant_q4_0(raw.ravel(), shape[0], shape[1]).astype(np.float64)

        self.audio = [emb(f"emb.{i}.weight") for i in range(meta["codebooks"])]
        self.text = emb("text_emb.weight")
        self.layers = []
        for l in range(meta["num_layers"]):
            p = f"transformer.layers.{l}."
            self.layers.append(dict(n1=norm(p + "norm1.alpha"), qkv=q4(p + "self_attn.in_proj_weight"),
                                    out=q4(p + "self_attn.out_proj.weight"), n2=norm(p + "norm2.alpha"),
                                    fin=q4(p + "gating.linear_in.weight"), fout=q4(p + "gating.linear_out.weight")))
        self.out_norm = norm("out_norm.alpha")
        self.head = q4("text_linear.weight")
        H = meta["heads"]
        self.H, self.HD, self.D = H, D // H, D
        half = self.HD // 2
        inv = 1.0 / (100000.0 ** (np.arange(half) * 2 / self.HD))
        self.inv = inv
        self.k = [[] for _ in self.layers]
        self.v = [[] for _ in self.layers]
        self.pos = 0

    @staticmethod
    def rms(x, a):
        return x / np.sqrt(np.mean(x * x) + 1e-8) * a

    def rope(self, x):
        c, s = np.cos(self.pos * self.inv), np.sin(self.pos * self.inv)
        x = x.reshape(self.H, self.HD // 2, 2)
        r, i = x[..., 0], x[..., 1]
        return np.stack([r * c - i * s, r * s + i * c], -1).reshape(-1)

    def forward(self, audio, text, window=750):
        x = sum(self.audio[i][a] for i, a in enumerate(audio)) + self.text[text]
        D, H, HD = self.D, self.H, self.HD
        for l, L in enumerate(self.layers):
            qkv = L["qkv"] @ self.rms(x, L["n1"])
            q, k, v = self.rope(qkv[:D]), self.rope(qkv[D:2 * D]), qkv[2 * D:]
            self.k[l].append(k)
            self.v[l].append(v)
            K = np.stack(self.k[l][-(window + 1):]).reshape(-1, H, HD)
            V = np.stack(self.v[l][-(window + 1):]).reshape(-1, H, HD)
            att = np.empty(D)
            for h in range(H):
                s = K[:, h] @ q[h * HD:(h + 1) * HD] / np.sqrt(HD)
                p = np.exp(s - s.max())
                att[h * HD:(h + 1) * HD] = (p / p.sum()) @ V[:, h]
            x = x + L["out"] @ att
            hcat = L["fin"] @ self.rms(x, L["n2"])
            F = hcat.size // 2
            g = hcat[:F]
            x = x + L["fout"] @ (g / (1 + np.exp(-g)) * hcat[F:])
        self.pos += 1
        return self.head @ self.rms(x, self.out_norm)


def test_oracle_forward_matches_float64_restatement(tiny_ref_gguf, tiny_meta):
    m = O.OracleModel(tiny_ref_gguf, num_layers=tiny_meta["num_layers"], num_heads=tiny_meta["heads"],
                      num_codebooks=tiny_meta["codebooks"], text_start_token=tiny_meta["text_vocab"] - 1)
    assert (m.hidden, m.ffn, m.vocab, m.text_vocab) == (tiny_meta["hidden"], tiny_meta["ffn"], tiny_meta["vocab"],
                                                       tiny_meta["text_vocab"])
    ref = F64Model(tiny_ref_gguf, tiny_meta)
    s = m.stream()
    rng = np.random.default_rng(11)
    text = tiny_meta["text_vocab"] - 1
    for step in range(8):
        audio = rng.integers(0, tiny_meta["audio_vocab"], tiny_meta["codebooks"])
        lg, am = s.forward(audio, text)
        r = ref.forward(audio, text)
        assert np.abs(lg - r).max() < 2e-4 * max(1.0, np.abs(r).max()), step
        text = am


def test_oracle_ring_wraps_like_reference(tiny_ref_gguf, tiny_meta):
    """sliding_window 5 -> ring of 6 slots; after wrapping, attention covers the last 6 steps."""
    m = O.OracleModel(tiny_ref_gguf, num_layers=tiny_meta["num_layers"], num_heads=tiny_meta["heads"],
                      num_codebooks=tiny_meta["codebooks"], text_start_token=tiny_meta["text_vocab"] - 1,
                      sliding_window=5)
    ref = F64Model(tiny_ref_gguf, tiny_meta)
    s = m.stream()
    rng = np.random.default_rng(5)
    for step in range(14):
        audio = rng.integers(0, tiny_meta["audio_vocab"], tiny_meta["codebooks"])
        lg, _ = s.forward(audio, 7)
        r = ref.forward(audio, 7, window=5)
        assert np.abs(lg - r).max() < 2e-4 * max(1.0, np.abs(r).max()), step
    st = s.state()
    assert (st["offset"], st["len"], st["write_pos"]) == (14, 6, 14 % 6)


def test_oracle_position_limit(tiny_ref_gguf, tiny_meta):
    m = O.OracleModel(tiny_ref_gguf, num_layers=tiny_meta["num_layers"], num_heads=tiny_meta["heads"],
                      num_codebooks=tiny_meta["codebooks"], text_start_token=tiny_meta["text_vocab"] - 1,
                      max_seq_len=3)
    s = m.stream()
    a = np.zeros(tiny_meta["codebooks"], np.uint32)
    for _ in range(3):
        s.forward(a, 0)
    with pytest.raises(RuntimeError, match="RoPE"):
        s.forward(a, 0)


def stream_rule(tokens, delay, pad=3, start=8000):
    """resolve_pending_as_token (stream.rs:231-266) over a sequence of argmax results.
    Returns (emitted per frame, text token fed to each frame)."""
    prev = [0xFFFFFFFF, 0xFFFFFFFF]
    last = start
    emitted, fed = [], []
    for i, tok in enumerate(tokens):
        fed.append(last)
        frame = i + 1
        if frame >= delay:
            last = tok
            emitted.append(tok)
        else:
            p0, p1 = prev
            prev = [p1, tok]
            last = pad if (tok != pad and tok != 0 and tok == p0 and tok != p1) else tok
            emitted.append(None)
    return emitted, fed


def test_oracle_feed_frame_follows_stream_rules(tiny_ref_gguf, tiny_meta):
    kw = dict(num_layers=tiny_meta["num_layers"], num_heads=tiny_meta["heads"], num_codebooks=tiny_meta["codebooks"],
              text_start_token=tiny_meta["text_vocab"] - 1)
    m = O.OracleModel(tiny_ref_gguf, **kw)
    a, b = m.stream(), m.stream()
    rng = np.random.default_rng(9)
    frames = rng.integers(0, tiny_meta["audio_vocab"], (20, tiny_meta["codebooks"]))
    got = [a.feed_frame(f) for f in frames]
    # replay with raw forwards, feeding back the text token the rule chooses
    toks, last = [], tiny_meta["text_vocab"] - 1
    prev = [0xFFFFFFFF] * 2
    for i, f in enumerate(frames):
        _, am = b.forward(f, last)
        toks.append(am)
        em, fed = stream_rule(toks, 6, start=tiny_meta["text_vocab"] - 1)
        last = em[-1] if em[-1] is not None else None
        if last is None:
            # the rule's choice for the next frame's text token
            p0, p1 = prev
            prev = [p1, am]
            last = 3 if (am != 3 and am != 0 and am == p0 and am != p1) else am
    em, _ = stream_rule(toks, 6, start=tiny_meta["text_vocab"] - 1)
    assert got == em
    assert got[:5] == [None] * 5 and all(t is not None for t in got[5:])
    fl = a.flush()
    assert len(fl) == 6


def test_stream_rule_limit_cycle_breaker():
    # A <-> B oscillation inside the delay: once the prediction repeats the one two frames back
    # (and differs from the last one), padding is fed instead; the history keeps the predictions
    em, fed = stream_rule([260, 263, 260, 263, 7, 8, 9], delay=6, start=8000)
    assert em == [None] * 5 + [8, 9]
    assert fed == [8000, 260, 263, 3, 3, 7, 8]
    # padding and 0 never trigger it
    em, fed = stream_rule([3, 5, 3, 0, 5, 0], delay=6, start=8000)
    assert fed == [8000, 3, 5, 3, 0, 5]

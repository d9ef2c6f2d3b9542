"""The oracle's batched step and the forward_with_gpu_token restatement.

A batch of streams in one oracle step must give every stream exactly (bit for bit) what it gets
stepped alone: the batched step is only a faster way to run the checker on many streams.

SttModel::forward_with_gpu_token (crates/stt-wasm/src/model.rs:675-722) adds the text row to the
finished 32-row audio sum, taking the row from the f32 table dequant_embedding_to_gpu builds
(gguf.rs:697-738); SttModel::forward (model.rs:631-664) adds the same row as the 33rd term of one
running sum.  Both orders are ((a0 + a1) + ... + a31) + t with t = (nibble - 8) * d computed the same
way, so the two paths give identical f32 values: the restatement of each is checked against the
other here, on the reference-converted checkpoint with Q4_0 embeddings."""
import numpy as np
import pytest

from oracle import oracle as O
import stt_b200

TINY = dict(num_layers=2, num_heads=2, num_codebooks=4, sliding_window=9)


def tiny_synth(seed, edt=30):
    spec = stt_b200.SynthSpec(seed=seed, num_layers=2, hidden_size=256, num_heads=2, ffn_hidden=512, vocab_size=1000,
                              text_in_vocab_size=1001, num_codebooks=4, audio_vocab_size=300, embedding_dtype=edt)
    return stt_b200.synth_gguf(spec)


@pytest.mark.parametrize("flags", [0, O.KV_BF16, O.GEMM_BF16])
def test_batched_step_equals_streams_alone(flags):
    g = tiny_synth(41)
    om = O.OracleModel(g.array, text_start_token=1000, **TINY)
    n = 5
    batch = [om.stream(flags) for _ in range(n)]
    alone = [om.stream(flags) for _ in range(n)]
    rng = np.random.default_rng(1)
    for s in range(n):                     # different positions, some past the ring size
        for _ in range(3 * s):
            a = rng.integers(0, 300, 4)
            batch[s].forward(a, 7)
            alone[s].forward(a, 7)
    texts = [1000] * n
    for step in range(6):
        audio = rng.integers(0, 300, (n, 4))
        lg, am = O.forward_batch(batch, audio, texts)
        for s in range(n):
            lo, ao = alone[s].forward(audio[s], texts[s])
            assert np.array_equal(lg[s].view(np.uint32), lo.view(np.uint32)), (step, s)
            assert am[s] == ao
        texts = [int(x) for x in am]


def test_batched_feed_frame_equals_feed_frame():
    g = tiny_synth(42)
    om = O.OracleModel(g.array, text_start_token=1000, **TINY)
    n = 4
    batch = [om.stream(O.KV_BF16) for _ in range(n)]
    alone = [om.stream(O.KV_BF16) for _ in range(n)]
    rng = np.random.default_rng(2)
    for f in range(12):
        audio = rng.integers(0, 300, (n, 4))
        toks, lg = O.feed_frame_batch(batch, audio, want_logits=True)
        assert toks == [alone[s].feed_frame(audio[s]) for s in range(n)]
        for s in range(n):
            assert batch[s].state() == alone[s].state()
    assert toks[0] is not None


def test_batched_step_rejects_bad_batches():
    g = tiny_synth(43)
    om = O.OracleModel(g.array, text_start_token=1000, **TINY)
    a, b = om.stream(), om.stream(O.KV_BF16)
    with pytest.raises(RuntimeError, match="share a model and flags"):
        O.forward_batch([a, b], np.zeros((2, 4)), [0, 0])
    with pytest.raises(RuntimeError, match="repeated"):
        O.forward_batch([a, a], np.zeros((2, 4)), [0, 0])
    with pytest.raises(RuntimeError, match="audio token"):
        O.forward_batch([a], np.full((1, 4), 300), [0])
    assert a.state()["offset"] == 0


@pytest.mark.parametrize("source", ["reference_converted", "q4_synthetic", "bf16_synthetic"])
def test_gpu_token_path_equals_forward(tiny_ref_gguf, source):
    if source == "reference_converted":
        buf = tiny_ref_gguf                # Q4_0 embeddings written by scripts/quantize.py
    else:
        buf = tiny_synth(44, edt=2 if source == "q4_synthetic" else 30).array
    om = O.OracleModel(buf, text_start_token=1000, **TINY)
    a5, a6 = om.stream(O.KV_BF16), om.stream(O.KV_BF16)
    rng = np.random.default_rng(3)
    prev = None
    text = 1000
    for f in range(15):
        audio = rng.integers(0, 300, 4)
        l5, t5 = a5.forward(audio, text)
        l6, t6 = a6.forward_gpu_token(audio, prev, 1000)   # no argmax yet on the first frame
        assert np.array_equal(l5.view(np.uint32), l6.view(np.uint32)), f
        assert t5 == t6
        prev, text = t6, t5

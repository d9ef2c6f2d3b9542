"""The decode step and the stream API on the GPU against the oracle.

Tolerances: the GPU computes in f32 like the reference but sums in a different order, so logits
agree to ~1e-5; the bound asserted is the task's 2e-2 max-abs, and argmax tokens must be equal
wherever the oracle's top-2 margin is not itself below 1e-3 (a genuine near-tie)."""
import numpy as np
import pytest

from oracle import oracle as O
import stt_b200
from stt_b200.model import SttConfig

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2
TIE = 1e-3


def tiny_cfg(**kw):
    c = SttConfig(num_layers=2, hidden_size=256, num_heads=2, num_kv_heads=2, num_codebooks=4,
                  text_start_token=1000, vocab_size=1000, text_in_vocab_size=1001, audio_vocab_size=300)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def oracle_for(buf, cfg: SttConfig):
    return O.OracleModel(buf, num_layers=cfg.num_layers, num_heads=cfg.num_heads, num_codebooks=cfg.num_codebooks,
                         text_start_token=cfg.text_start_token, text_delay=cfg.text_delay,
                         max_seq_len=cfg.max_seq_len, sliding_window=cfg.sliding_window)


def margin(lg):
    s = np.sort(lg)
    return s[-1] - s[-2]


def compare_steps(model, cache, om, flags, frames, text0, stream_id=0):
    """Teacher-forced raw steps; returns the max logit difference seen."""
    os_ = om.stream(flags)
    text = text0
    worst = 0.0
    for f in frames:
        lg_o, am_o = os_.forward(f, text)
        lg_g = model.forward(f, text, cache, stream_id).reshape(-1)
        d = float(np.abs(lg_g - lg_o).max())
        worst = max(worst, d)
        assert d < LOGIT_TOL, d
        if margin(lg_o) > TIE:
            assert int(np.argmax(lg_g)) == am_o
        text = am_o
    return worst


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_tiny_reference_checkpoint_steps(tiny_ref_gguf, kv):
    cfg = tiny_cfg()
    model = stt_b200.SttModel.from_shards([tiny_ref_gguf], config=cfg)
    assert model.info.embedding_dtype == 2  # quantize.py writes Q4_0 embeddings
    cache = model.create_cache(1, kv)
    om = oracle_for(tiny_ref_gguf, cfg)
    frames = np.random.default_rng(1).integers(0, 300, (24, 4))
    worst = compare_steps(model, cache, om, 0 if kv == "f32" else O.KV_BF16, frames, 1000)
    assert worst < 1e-3, worst


def test_ring_wraps(tiny_ref_gguf):
    cfg = tiny_cfg(sliding_window=9)
    model = stt_b200.SttModel.from_shards([tiny_ref_gguf], config=cfg)
    cache = model.create_cache(1, "f32")
    om = oracle_for(tiny_ref_gguf, cfg)
    frames = np.random.default_rng(2).integers(0, 300, (31, 4))
    compare_steps(model, cache, om, 0, frames, 1000)
    st = cache.state(0)
    assert (st["offset"], st["len"], st["write_pos"]) == (31, 10, 31 % 10)


@pytest.mark.parametrize("edt", [30, 2])
def test_stream_api_matches_oracle(edt):
    spec = stt_b200.SynthSpec(seed=21, num_layers=2, hidden_size=256, num_heads=2, ffn_hidden=512, vocab_size=1000,
                              text_in_vocab_size=1001, num_codebooks=4, audio_vocab_size=300, embedding_dtype=edt)
    g = stt_b200.synth_gguf(spec)
    cfg = tiny_cfg()
    model = stt_b200.SttModel.from_shards([g.array], config=cfg)
    cache = model.create_cache(2, "bf16")
    om = oracle_for(g.array, cfg)
    ref = om.stream(O.KV_BF16)
    st = stt_b200.SttStream(cfg, cache, stream_id=1)
    frames = np.random.default_rng(3).integers(0, 300, (20, 4))
    got = [st.feed_frame(f, model) for f in frames]
    exp = [ref.feed_frame(f) for f in frames]
    assert got == exp
    assert got[:5] == [None] * 5
    assert st.flush(model) == ref.flush()
    s = cache.state(1)
    r = ref.state()
    assert (s["offset"], s["len"], s["write_pos"], s["frame_count"], s["last_text_token"]) == \
           (r["offset"], r["len"], r["write_pos"], r["frame_count"], r["last_text_token"])
    # stream 0 was never touched
    assert cache.state(0)["offset"] == 0
    # reset: identical to a fresh stream
    st.reset_keep_buffers()
    ref.reset()
    assert [st.feed_frame(f) for f in frames[:8]] == [ref.feed_frame(f) for f in frames[:8]]
    st.reset()
    ref.reset()
    st.set_last_text_token(17)
    ref.set_last_text_token(17)
    assert [st.feed_frame(f) for f in frames[:8]] == [ref.feed_frame(f) for f in frames[:8]]


def test_feed_frames_equals_feed_frame_loop():
    spec = stt_b200.SynthSpec(seed=22, num_layers=2, hidden_size=256, num_heads=2, ffn_hidden=512, vocab_size=1000,
                              text_in_vocab_size=1001, num_codebooks=4, audio_vocab_size=300)
    g = stt_b200.synth_gguf(spec)
    cfg = tiny_cfg()
    model = stt_b200.SttModel.from_shards([g.array], config=cfg)
    cache = model.create_cache(2, "bf16")
    a = stt_b200.SttStream(cfg, cache, 0)
    b = stt_b200.SttStream(cfg, cache, 1)
    frames = np.random.default_rng(4).integers(0, 300, (40, 4))
    one = [a.feed_frame(f) for f in frames]
    many = b.feed_frames(frames)
    assert one == many


def test_batched_streams_at_staggered_positions():
    spec = stt_b200.SynthSpec(seed=23, num_layers=2, hidden_size=256, num_heads=2, ffn_hidden=512, vocab_size=1000,
                              text_in_vocab_size=1001, num_codebooks=4, audio_vocab_size=300)
    g = stt_b200.synth_gguf(spec)
    cfg = tiny_cfg(sliding_window=12)
    model = stt_b200.SttModel.from_shards([g.array], config=cfg)
    n = 5
    cache = model.create_cache(n, "bf16")
    om = oracle_for(g.array, cfg)
    refs = [om.stream(O.KV_BF16) for _ in range(n)]
    rng = np.random.default_rng(5)
    # pre-roll stream s by 3*s frames on its own
    for s in range(n):
        for _ in range(3 * s):
            f = rng.integers(0, 300, 4)
            model.forward(f, 5, cache, s)
            refs[s].forward(f, 5)
    order = [3, 0, 4, 1, 2]
    texts = [1000] * n
    for step in range(10):
        audio = rng.integers(0, 300, (n, 4))
        lg, am = cache.forward(order, audio, [texts[s] for s in order])
        for i, s in enumerate(order):
            lo, ao = refs[s].forward(audio[i], texts[s])
            assert np.abs(lg[i] - lo).max() < 1e-3
            if margin(lo) > TIE:
                assert am[i] == ao
            texts[s] = ao


def test_errors_raised_where_the_reference_panics(tiny_ref_gguf):
    cfg = tiny_cfg(max_seq_len=4)
    model = stt_b200.SttModel.from_shards([tiny_ref_gguf], config=cfg)
    cache = model.create_cache(2)
    ok = np.zeros(4, np.uint32)
    with pytest.raises(stt_b200.SttError, match="audio token 300"):
        model.forward(np.array([0, 0, 300, 0]), 0, cache)
    with pytest.raises(stt_b200.SttError, match="text token 1001"):
        model.forward(ok, 1001, cache)
    with pytest.raises(stt_b200.SttError, match="out of range"):
        model.forward(ok, 0, cache, stream_id=2)
    with pytest.raises(stt_b200.SttError, match="repeated"):
        cache.forward([1, 1], np.zeros((2, 4)), [0, 0])
    for _ in range(4):
        model.forward(ok, 0, cache)
    with pytest.raises(stt_b200.SttError) as e:
        model.forward(ok, 0, cache)
    assert e.value.code == -6
    assert cache.state(0)["offset"] == 4 and cache.state(1)["offset"] == 0


@pytest.fixture(scope="module")
def full_model():
    g = stt_b200.synth_gguf()
    model = stt_b200.SttModel.from_shards([g.array])
    yield g, model
    model.close()


@pytest.mark.parametrize("kv,bound", [("f32", 1e-3), ("bf16", LOGIT_TOL)])
def test_full_size_model_parity(full_model, kv, bound):
    """Raw steps (n = 1: the persistent kernel) against the oracle at the full model size.  With
    bf16 K/V a 1e-6 difference can flip a bf16 rounding of K or V, so that mode is held to the
    2e-2 bound; f32 K/V is held to 1e-3."""
    g, model = full_model
    assert model.info.q4_weight_bytes == 627_351_552
    cache = model.create_cache(1, kv)
    om = oracle_for(g.array, SttConfig())
    frames = stt_b200.audio_tokens(1, 0, 6)
    worst = compare_steps(model, cache, om, 0 if kv == "f32" else O.KV_BF16, frames, 0)
    assert worst < bound, worst


def test_full_size_feed_frame_tokens_identical(full_model):
    g, model = full_model
    cache = model.create_cache(1, "bf16")
    cfg = SttConfig()
    st = stt_b200.SttStream(cfg, cache)
    ref = oracle_for(g.array, cfg).stream(O.KV_BF16)
    frames = stt_b200.audio_tokens(2, 0, 10)
    assert st.feed_frames(frames) == [ref.feed_frame(f) for f in frames]


def test_persistent_kernel_and_graph_path_agree(full_model, monkeypatch):
    """The single-stream persistent kernel and the multi-kernel graph path decode the same
    utterance to the same tokens."""
    g, model = full_model
    cfg = SttConfig()
    frames = stt_b200.audio_tokens(3, 0, 40)
    a = model.create_cache(1, "bf16")
    toks_mega = stt_b200.SttStream(cfg, a).feed_frames(frames)
    monkeypatch.setenv("STT_DISABLE_MEGA", "1")
    b = model.create_cache(1, "bf16")
    toks_graph = stt_b200.SttStream(cfg, b).feed_frames(frames)
    monkeypatch.delenv("STT_DISABLE_MEGA")
    assert toks_mega == toks_graph
    sa, sb = a.state(0), b.state(0)
    assert sa == sb and sa["offset"] == 40


def test_persistent_kernel_barrier_and_trace(full_model):
    import ctypes as C
    from stt_b200._lib import lib
    ns = C.c_double()
    for mode in (0, 1):
        assert lib().stt_debug_barrier_ns(0, 2000, mode, C.byref(ns)) == 0
        assert 50 < ns.value < 20000, ns.value
    g, model = full_model
    cache = model.create_cache(1, "bf16")
    assert lib().stt_debug_trace_frame(cache._h, 1) == 0
    stt_b200.SttStream(SttConfig(), cache).feed_frames(stt_b200.audio_tokens(4, 0, 3))
    buf = (C.c_uint64 * 1024)()
    n = C.c_int()
    assert lib().stt_debug_get_trace(cache._h, buf, 1024, C.byref(n)) == 0
    # (tag, time) pairs: frame start; per layer 3 marks for each of the 4 GEMV phases and 4 for
    # attention (CTA 0 merges the splits of head 0); the head's 3 marks and the argmax
    tags = list(buf[0:n.value:2])
    marks = [i for i, t in enumerate(tags) if 0 < t < 100]  # tags >= 100 carry wait durations
    assert len(marks) == 1 + 16 * (4 * 3 + 4) + 3 + 1, len(marks)
    assert tags[0] == 0 and tags[-1] == 0  # wall-clock pairs around the frame
    t = np.array([buf[2 * i + 1] for i in marks], dtype=np.int64)
    assert np.all(np.diff(t) >= 0)


TC_TIE = 5e-2  # near-ties below this margin may flip under f16 operand rounding


@pytest.mark.parametrize("kv,n", [("bf16", 20), ("f32", 20), ("bf16", 40), ("bf16", 100), ("bf16", 150),
                                  ("bf16", 260), ("f32", 260)])
def test_batched_tensor_core_path_matches_oracle(tiny_ref_gguf, kv, n):
    """Batches of 16+ streams run their layer products on the tensor cores (f16 operand parts,
    K-slice partial sums added in order; 20, 40, 100 and 150 streams take batch tiles of 32, 64,
    128 and 256 rows, 260 streams two 256-row tiles and the attention's 32-key K/V chunks): logits
    within the 2e-2 bound of the oracle, tokens equal away from near-ties."""
    cfg = tiny_cfg(sliding_window=12)
    model = stt_b200.SttModel.from_shards([tiny_ref_gguf], config=cfg)
    assert model.info.tensor_core_min_batch == 16
    cache = model.create_cache(n, kv)
    om = oracle_for(tiny_ref_gguf, cfg)
    refs = [om.stream(0 if kv == "f32" else O.KV_BF16) for _ in range(n)]
    rng = np.random.default_rng(9)
    for s in range(n):  # staggered positions, some past the ring size
        for _ in range(s % 7 + (s // 7) * 6):
            f = rng.integers(0, 300, 4)
            model.forward(f, 5, cache, s)
            refs[s].forward(f, 5)
    order = list(rng.permutation(n))
    texts = [1000] * n
    worst = 0.0
    for step in range(8):
        audio = rng.integers(0, 300, (n, 4))
        lg, am = cache.forward(order, audio, [texts[s] for s in order])
        for i, s in enumerate(order):
            lo, ao = refs[s].forward(audio[i], texts[s])
            worst = max(worst, float(np.abs(lg[i] - lo).max()))
            if margin(lo) > TC_TIE:
                assert am[i] == ao
            texts[s] = ao
    assert worst < LOGIT_TOL, worst


def test_full_size_batched_tensor_core_path(full_model):
    g, model = full_model
    assert model.info.tensor_core_min_batch == 16
    n = 16
    cache = model.create_cache(n, "bf16")
    om = oracle_for(g.array, SttConfig())
    refs = [om.stream(O.KV_BF16) for _ in range(n)]
    ids = list(range(n))
    texts = [0] * n
    worst = 0.0
    for step in range(3):
        audio = np.stack([stt_b200.audio_tokens(11, s, 1, first_frame=step)[0] for s in ids])
        lg, am = cache.forward(ids, audio, texts)
        for s in ids:
            lo, ao = refs[s].forward(audio[s], texts[s])
            worst = max(worst, float(np.abs(lg[s] - lo).max()))
            if margin(lo) > TC_TIE:
                assert am[s] == ao
            texts[s] = ao
    assert worst < LOGIT_TOL, worst


@pytest.mark.parametrize("n", [20, 150])
def test_gate_fused_into_linear_in_is_bit_identical(monkeypatch, n):
    """linear_in with the SiLU gate in its epilogue (writing the linear_out input directly) gives
    the same logits, bit for bit, as linear_in followed by the separate gate kernel."""
    spec = stt_b200.SynthSpec(seed=25, num_layers=2, hidden_size=256, num_heads=2, ffn_hidden=512, vocab_size=1000,
                              text_in_vocab_size=1001, num_codebooks=4, audio_vocab_size=300)
    g = stt_b200.synth_gguf(spec)
    model = stt_b200.SttModel.from_shards([g.array], config=tiny_cfg())
    frames = np.random.default_rng(13).integers(0, 300, (5, n, 4))
    outs = []
    for unfused in (False, True):
        if unfused:
            monkeypatch.setenv("STT_UNFUSED_GATE", "1")
        cache = model.create_cache(n, "bf16")
        texts = [1000] * n
        lgs = []
        for f in frames:
            lg, am = cache.forward(list(range(n)), f, texts)
            lgs.append(lg)
            texts = [int(t) for t in am]
        outs.append(np.stack(lgs))
        cache.close()
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


def test_tensor_core_and_gemv_batches_agree(monkeypatch):
    """The same 16-stream batch through the tensor cores and through the GEMV (STT_DISABLE_TC)."""
    spec = stt_b200.SynthSpec(seed=24, num_layers=2, hidden_size=256, num_heads=2, ffn_hidden=512, vocab_size=1000,
                              text_in_vocab_size=1001, num_codebooks=4, audio_vocab_size=300)
    g = stt_b200.synth_gguf(spec)
    cfg = tiny_cfg()
    model = stt_b200.SttModel.from_shards([g.array], config=cfg)
    assert model.info.tensor_core_min_batch == 16
    n = 16
    frames = np.random.default_rng(12).integers(0, 300, (6, n, 4))
    outs = []
    for disable in (False, True):
        if disable:
            monkeypatch.setenv("STT_DISABLE_TC", "1")
        cache = model.create_cache(n, "bf16")
        toks, lgs = [], []
        texts = [1000] * n
        for f in frames:
            lg, am = cache.forward(list(range(n)), f, texts)
            lgs.append(lg)
            toks.append(list(am))
            texts = [int(a) for a in am]
        outs.append((toks, np.stack(lgs)))
        cache.close()
    monkeypatch.delenv("STT_DISABLE_TC")
    assert np.abs(outs[0][1] - outs[1][1]).max() < LOGIT_TOL


def test_bounded_wait_runs_out_and_the_next_call_recovers():
    """A persistent-kernel wait that nothing will satisfy gives up after its limit: the call returns
    STT_E_DEVICE_FLAG within seconds instead of hanging, and the stream set stays usable: after a
    reset the same frames decode exactly as the oracle's."""
    import ctypes as C
    import time
    from stt_b200._lib import lib, STT_E_DEVICE_FLAG
    spec = stt_b200.SynthSpec(seed=25, num_layers=2, hidden_size=256, num_heads=2, ffn_hidden=512, vocab_size=1000,
                              text_in_vocab_size=1001, num_codebooks=4, audio_vocab_size=300)
    g = stt_b200.synth_gguf(spec)
    cfg = tiny_cfg()
    model = stt_b200.SttModel.from_shards([g.array], config=cfg)
    cache = model.create_cache(1, "bf16")
    st = stt_b200.SttStream(cfg, cache)
    frames = np.random.default_rng(6).integers(0, 300, (10, 4))
    assert lib().stt_debug_arm_wait_timeout(cache._h) == 0
    t0 = time.perf_counter()
    with pytest.raises(stt_b200.SttError) as e:
        st.feed_frames(frames[:3])
    took = time.perf_counter() - t0
    assert e.value.code == STT_E_DEVICE_FLAG, e.value
    assert took < 30.0, took
    assert cache.state(0)["offset"] == 0          # the failed frame changed no stream state
    st.reset()
    ref = oracle_for(g.array, cfg).stream(O.KV_BF16)
    assert st.feed_frames(frames) == [ref.feed_frame(f) for f in frames]
    # the hook was one-shot: a second call runs normally too
    assert st.feed_frame(frames[0]) == ref.feed_frame(frames[0])


def test_allocation_failures_release_everything():
    """An allocation that fails part-way through loading a model, creating a stream set or a step's
    first use of its staging buffers is reported as STT_E_OOM, and whatever the call had already
    allocated is released: after each failure, device memory is back where it started, and a later
    attempt succeeds and decodes like the oracle.  (The failure is injected on the host, where the
    library asks for memory.)"""
    import torch
    from stt_b200._lib import lib, STT_E_OOM
    spec = stt_b200.SynthSpec(seed=26, num_layers=2, hidden_size=256, num_heads=2, ffn_hidden=512, vocab_size=1000,
                              text_in_vocab_size=1001, num_codebooks=4, audio_vocab_size=300)
    g = stt_b200.synth_gguf(spec)
    cfg = tiny_cfg()
    frames = np.random.default_rng(10).integers(0, 300, (3, 20, 4))
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    failures = 0
    for k in range(40):
        assert lib().stt_debug_fail_allocation(k) == 0
        model = cache = None
        try:
            model = stt_b200.SttModel.from_shards([g.array], config=cfg)
            cache = model.create_cache(20, "bf16")
            toks = [cache.feed_frame(list(range(20)), f) for f in frames]
            ok = True
        except stt_b200.SttError as e:
            assert e.code == STT_E_OOM, e
            ok = False
            failures += 1
        finally:
            lib().stt_debug_fail_allocation(-1)
            if cache is not None:
                cache.close()
            if model is not None:
                model.close()
        torch.cuda.synchronize()
        assert abs(torch.cuda.mem_get_info()[0] - free0) < (64 << 20), k
        if ok:
            break
    assert failures >= 3 and ok
    om = oracle_for(g.array, cfg)
    refs = [om.stream(O.KV_BF16) for _ in range(20)]
    exp = [O.feed_frame_batch(refs, f)[0] for f in frames]
    assert [[None if t < 0 else int(t) for t in row] for row in toks] == exp

"""The roofline arithmetic of bench.py: byte and FLOP counts against the model's shapes."""
import importlib.util
import os

import pytest

REPO = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..")


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def q4_bytes(n, k):
    return n * k // 32 * 18


def test_weight_bytes_and_params(bench):
    # 16 x (in_proj 6144x2048, out_proj 2048x2048, linear_in 16896x2048, linear_out 2048x8448) + head 8000x2048
    layer = [(6144, 2048), (2048, 2048), (16896, 2048), (2048, 8448)]
    params = 16 * sum(n * k for n, k in layer) + 8000 * 2048
    assert bench.Q4_PARAMS == params == 1_115_291_648
    assert bench.WEIGHT_BYTES == 16 * sum(q4_bytes(n, k) for n, k in layer) + q4_bytes(8000, 2048)
    assert bench.KV_BYTES_PER_TOKEN == 131_072


def test_bytes_per_utterance(bench):
    # 750 frames from position 0: weights and embeddings every frame, K/V of positions 0..t read at t
    total = bench.algorithmic_bytes_per_utterance(750)
    assert total == 750 * (bench.WEIGHT_BYTES + bench.EMB_BYTES) + (sum(range(1, 751)) + 750) * 131_072
    assert abs(total / 750 / 1e6 - 676.8) < 0.1  # MB per frame


def test_bytes_per_batched_step(bench):
    # configuration 3: stream s pre-rolled to round(374 s / 63); 375 steps, 3 of them warm-up
    offs = [round(s * 374 / 63) for s in range(64)]
    per_step = bench.algorithmic_bytes_batched(offs, 3, 375)
    assert 3.7e9 < per_step < 3.9e9
    # one step of one stream at position p reads p + 1 slots and writes one
    one = bench.algorithmic_bytes_batched([10], 0, 1)
    assert one == bench.WEIGHT_BYTES + (11 + 1) * 131_072 + bench.EMB_BYTES
    # the ring caps the slots read at 751
    assert bench.algorithmic_bytes_batched([2000], 0, 1) == bench.WEIGHT_BYTES + (751 + 1) * 131_072 + bench.EMB_BYTES


def test_both_arms_describe_one_workload(bench):
    # the GPU arm and the reference arm print the same config object for a given GPU count
    for n in (1, 2, 4, 8):
        c = bench.job_config(n)
        assert c == bench.job_config(n)
        assert c["streams"] == 512 and c["frames_per_stream"] == 250
        assert f"{512 // n} streams" in c["parallelism"]


def test_reference_arm_loads_no_decode_library(tmp_path):
    """--impl reference runs the oracle on a bounded sample of the job and maps no library of the
    decode path (the synthetic checkpoint comes from the separate generator library)."""
    import json
    import subprocess
    import sys
    env = dict(os.environ, OMP_NUM_THREADS="1")   # as torchrun sets it: the arm must override it
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], capture_output=True, text=True, env=env, timeout=600, check=True).stdout
    line = json.loads(out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["steps"] == 1 and line["warmup"] == 0
    assert line["config"] == json.loads(json.dumps(_bench_module().job_config(1)))
    assert line["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0)) > 0
    libs = line["libraries"]
    assert "oracle/liboracle.so" in libs
    assert all(x.startswith("oracle/") for x in libs), libs   # nothing of the decode package
    # the timed steps fit the run: ms_per_step x steps is the sample's own time
    assert 0 < line["ms_per_step"] < 600_000


def _bench_module():
    spec = importlib.util.spec_from_file_location("bench_under_test2", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_both_generator_builds_write_the_same_checkpoint():
    """The oracle's build of the generator (oracle/libsynth.so, for the CPU baseline) and the
    package's (libsttsynth.so) are one source with one set of flags: byte-identical output."""
    import ctypes as C
    import numpy as np
    from stt_b200 import synth
    spec = synth.SynthSpec(seed=9, num_layers=2, hidden_size=256, num_heads=2, ffn_hidden=512, vocab_size=1000,
                           text_in_vocab_size=1001, num_codebooks=4, audio_vocab_size=300, embedding_dtype=2)
    outs = []
    for path in (synth.SYNTH_LIB_PATH, os.path.join(REPO, "oracle", "libsynth.so")):
        L = C.CDLL(path)
        L.stt_synth_gguf.argtypes = [C.POINTER(synth.stt_synth_params), C.POINTER(C.POINTER(C.c_uint8)),
                                     C.POINTER(C.c_size_t)]
        L.stt_synth_free.argtypes = [C.POINTER(C.c_uint8)]
        p = spec.to_c()
        ptr, n = C.POINTER(C.c_uint8)(), C.c_size_t()
        assert L.stt_synth_gguf(C.byref(p), C.byref(ptr), C.byref(n)) == 0
        outs.append(np.ctypeslib.as_array(ptr, shape=(n.value,)).copy())
        L.stt_synth_free(ptr)
    assert np.array_equal(outs[0], outs[1])

#!/usr/bin/env python
"""Decode throughput of the STT-1B Q4 decode step on B200.

Headline workload (one bench step): 512 independent streams each decode 250 frames from position 0
(configuration 4), split into contiguous blocks of global stream ids over the N GPUs (one process
per GPU, no collective on the data path: strong scaling, the whole job is fixed).  Model: the full
STT-1B (16 layers, d_model 2048, 16 x 128 heads, FFN 8448, Q4_0 linear weights of 627,351,552 bytes
per step, bf16 embeddings and norms), seeded synthetic weights N(0, 0.02); seeded uniform audio
tokens in [0, 2048); initial text token 0; the feed_frame loop (text delay, limit-cycle rule) with
greedy tokens fed back on the device; bf16 K/V.

  value     whole-job frames/s with the audio tokens already in HBM: device time (CUDA events on the
            launch stream) of K steps, max over ranks
  e2e       the same job through the public host-buffer call stt_streams_feed_frame (host audio in,
            host tokens out, one call per batched frame), host wall clock, max over ranks
  roofline  the dominant kernel of that step, the tcgen05 Q4 GEMM: useful FLOPs per launch over its
            CUDA-event launch time, against the measured bf16 tensor peak
  stream1   configuration 2: one stream decodes a 750-frame utterance (the persistent kernel)
  streams64 configuration 3: 64 streams per GPU at staggered offsets 0..374, 375 batched steps
  q4_matmul configuration 5: the isolated Q4_0 matmul sweep
  --impl reference  the CPU restatement of the reference step (oracle/) on the host cores, on a
            bounded sample of the headline workload; it loads no library of the decode path
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(REPO, "stt-web_b200"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

SEED = 0x5EED5EED
JOB_STREAMS = 512                # configuration 4: 512 streams ...
JOB_FRAMES = 250                 # ... x 250 frames each, from position 0
UTT_FRAMES = 750                 # configuration 2: one 750-frame utterance (the full window)
WEIGHT_BYTES = 627_351_552       # Q4_0 bytes of all linear layers, read once per step
KV_BYTES_PER_TOKEN = 16 * 2 * 2048 * 2   # bf16 K+V of one cached position over 16 layers
EMB_BYTES = 33 * 2048 * 2        # 33 bf16 embedding rows per frame
# Q4_0 weights of one step (16 layers + head): useful work is 2 FLOPs per weight per stream row
Q4_PARAMS = 16 * (6144 * 2048 + 2048 * 2048 + 16896 * 2048 + 2048 * 8448) + 8000 * 2048
# The reference's published 1-stream step time over a 750-frame (60 s) utterance: 52.5 ms per frame
# on an Apple M2 GPU through wgpu/Metal (BENCHMARKS.md:29 of stt-web).
PUBLISHED_FPS_750 = 1000.0 / 52.5
# DRAM read + write bytes of one 750-frame launch of the persistent kernel (ncu, single pass):
# profiles/mega_kernel_dram_750frames.txt
MEGA_TRAFFIC_750 = 508_170_845_440 + 2_636_432_128
# DRAM read + write bytes of one launch of the tcgen05 GEMM on linear_in (16896 x 2048) at 512 batch
# rows (ncu): profiles/q4_tc_kernel_linear_in_512rows.txt
TC_TRAFFIC_LINEAR_IN_512 = 23_695_360 + 194_048
METRIC = "decode frames/s, whole job (512 streams x 250 frames split over the GPUs)"


def job_config(n_gpus):
    """The `config` object of both arms (identical, so the two lines describe one workload)."""
    per = JOB_STREAMS // n_gpus
    return {"workload": f"{JOB_STREAMS} independent streams x {JOB_FRAMES} frames from position 0, "
                        f"STT-1B Q4_0 (16 layers, d_model 2048), greedy feed_frame loop, bf16 KV",
            "streams": JOB_STREAMS, "frames_per_stream": JOB_FRAMES,
            "parallelism": f"{n_gpus} GPU(s) x {per} streams, contiguous blocks of stream ids, no collective",
            "l2": "inputs larger than L2: 627 MB of Q4 weights and the K/V rings streamed every step"}


def algorithmic_bytes_per_utterance(frames=UTT_FRAMES, ring=751):
    kv_read = sum(min(p + 1, ring) for p in range(frames)) * KV_BYTES_PER_TOKEN
    kv_write = frames * KV_BYTES_PER_TOKEN
    return frames * (WEIGHT_BYTES + EMB_BYTES) + kv_read + kv_write


def algorithmic_bytes_batched(offsets, first, last, ring=751):
    """Mean algorithmic bytes of the batched steps first .. last-1: the weights once per step, each
    stream's K/V reads at its position (offset + step), its K/V write and its 33 embedding rows."""
    total = 0
    for f in range(first, last):
        total += WEIGHT_BYTES + sum((min(o + f + 1, ring) + 1) * KV_BYTES_PER_TOKEN + EMB_BYTES for o in offsets)
    return total / max(1, last - first)


def peaks():
    try:
        return json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json"))), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def loaded_libraries():
    """Shared libraries of this repository that the process has mapped (from /proc/self/maps)."""
    out = set()
    try:
        for line in open("/proc/self/maps"):
            path = line.split()[-1] if len(line.split()) >= 6 else ""
            if path.endswith(".so") and path.startswith(REPO):
                out.add(os.path.relpath(path, REPO))
    except OSError:
        pass
    return sorted(out)


TRACE_NAMES = {1: "frame_start", 11: "qkv_inputs", 12: "qkv_gemv", 13: "qkv_end", 21: "attention_inputs",
               22: "attention", 24: "attention_merge", 23: "attention_end", 31: "out_proj_inputs",
               32: "out_proj_gemv", 33: "out_proj_end", 41: "linear_in_inputs", 42: "linear_in_gemv",
               43: "linear_in_end", 51: "linear_out_inputs", 52: "linear_out_gemv", 53: "linear_out_end",
               61: "head_inputs", 62: "head_gemv", 63: "head_partial", 7: "argmax"}
LAYER_TAGS = [11, 12, 13, 21, 22, 24, 23, 31, 32, 33, 41, 42, 43, 51, 52, 53]
HEAD_TAGS = [61, 62, 63, 7]


def critical_path(buf, n_ctas, n_slots, layers):
    """Every CTA's %globaltimer stamps of one traced frame of the persistent kernel -> how far the
    latest CTA moves at each kind of mark (the frame's critical path), in microseconds per frame."""
    import numpy as np
    t = np.array(buf, dtype=np.int64).reshape(n_ctas, n_slots)
    starts = t[:, 0][t[:, 0] > 0]
    if starts.size == 0:
        return {}
    order = [(1 + 16 * l + i, tag) for l in range(layers) for i, tag in enumerate(LAYER_TAGS)]
    order += [(1 + 16 * layers + i, tag) for i, tag in enumerate(HEAD_TAGS)]
    prev = int(starts.max())
    crit = {}
    last = prev
    for slot, tag in order:
        v = t[:, slot][t[:, slot] > 0]
        if v.size == 0:
            continue
        mx = int(v.max())
        name = TRACE_NAMES.get(tag, str(tag))
        crit[name] = crit.get(name, 0.0) + (mx - prev) / 1e3
        prev = mx
        last = mx
    return {"frame_us_all_ctas": round((last - int(starts.min())) / 1e3, 1),
            "critical_path_us": {k: round(v, 1) for k, v in crit.items()}}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(5)
            except Exception:
                self.p.kill()

    def summary(self):
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if "Active" in v and "Not" not in v:
                        reasons.add(n)
            except Exception:
                pass
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------ CPU arm

class CpuJob:
    """A bounded sample of the headline workload on the CPU restatement of the reference step
    (oracle/, reference f32 arithmetic with the K/V rounded to bf16 as the job stores it): the
    first `streams` streams of the job, batched per matmul, advancing `frames` frames per step
    from position 0 (back to position 0 after frame 250, as the job does)."""

    def __init__(self, streams=16, frames=2):
        from oracle import oracle as O
        from stt_b200 import synth   # the generator's Python wrapper only: no decode library is loaded
        if synth._slib is None:      # the oracle's own build of the generator (same source and flags)
            synth.SYNTH_LIB_PATH = os.path.join(REPO, "oracle", "libsynth.so")
        self.O = O
        self.cores = len(os.sched_getaffinity(0))
        O.set_threads(self.cores)    # torchrun sets OMP_NUM_THREADS=1; the baseline uses every core
        self.g = synth.synth_gguf(synth.SynthSpec(seed=SEED, n_threads=self.cores))
        self.model = O.OracleModel(self.g.array, text_start_token=0)
        self.n, self.frames = streams, frames
        self.streams = [self.model.stream(O.KV_BF16) for _ in range(streams)]
        self.audio = __import__("numpy").stack([synth.audio_tokens(SEED, s, JOB_FRAMES) for s in range(streams)], 1)
        self.pos = 0

    def step(self):
        for _ in range(self.frames):
            if self.pos == JOB_FRAMES:
                for s in self.streams:
                    s.reset()
                self.pos = 0
            self.O.feed_frame_batch(self.streams, self.audio[self.pos])
            self.pos += 1
        return self.n * self.frames

    def sample(self):
        return (f"streams 0..{self.n - 1} of the job, {self.frames} frames each per step (positions 0..249 in "
                f"turn), one batched oracle step per frame, f32 arithmetic, bf16 K/V")


def run_reference(args):
    """--impl reference: times the oracle on the host cores, rank 0 only (other ranks exit)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    job = CpuJob()
    for _ in range(args.warmup):
        job.step()
    t0 = time.perf_counter()
    frames = 0
    for _ in range(args.steps):
        frames += job.step()
    dt = time.perf_counter() - t0
    fps = frames / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": fps, "unit": "frames/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1000.0 / max(1, args.steps),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": job_config(args.gpus),
        "cpu_baseline": {"value": fps, "unit": "frames/s", "cores": job.cores, "kind": "port", "sample": job.sample()},
        "e2e": {"value": fps, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "libraries": loaded_libraries(),
    }
    print(json.dumps(line))
    return 0


# ------------------------------------------------------------------------------------ GPU arm

def batched_job(model, cache, S, frames, da, dt, lib, check, ts):
    """One step of a batched job on this GPU: every stream of the set back to position 0, then
    `frames` batched feed_frame steps of all S streams with device-resident audio and tokens."""
    ids = (C.c_int32 * S)(*range(S))
    for s in range(S):
        check(lib().stt_stream_reset_async(cache._h, s, 0, C.c_void_p(ts.cuda_stream)), "reset_async")
    for f in range(frames):
        check(lib().stt_streams_feed_frame_device(cache._h, ids, S, C.c_void_p(da[f].data_ptr()),
                                                  C.c_void_p(dt[f].data_ptr()), C.c_void_p(ts.cuda_stream)), "step")


def staggered(model, stream_ids, F, offsets, seed, torch, np, lib, check, synth):
    """Configuration 3 on this GPU: the S streams of those global ids, the s-th pre-rolled alone to
    offsets[s] frames, then F batched steps of all S streams, device-timed (the last F - 3)."""
    S = len(stream_ids)
    cache = model.create_cache(S, "bf16")
    ts = torch.cuda.current_stream()
    for s_ in range(S):
        if offsets[s_]:
            pre = synth.audio_tokens(seed, stream_ids[s_], offsets[s_])
            a = torch.from_numpy(pre.astype(np.int32)).cuda()
            tk = torch.empty(offsets[s_], dtype=torch.int32, device="cuda")
            check(lib().stt_stream_feed_frames_device(cache._h, s_, offsets[s_], C.c_void_p(a.data_ptr()),
                                                      C.c_void_p(tk.data_ptr()), C.c_void_p(ts.cuda_stream)), "pre-roll")
    aud = np.stack([synth.audio_tokens(seed, stream_ids[s_], F, first_frame=offsets[s_]) for s_ in range(S)], 1)
    da = torch.from_numpy(aud.astype(np.int32)).cuda()
    dt = torch.empty(F, S, dtype=torch.int32, device="cuda")
    ids = (C.c_int32 * S)(*range(S))

    def step(f):
        check(lib().stt_streams_feed_frame_device(cache._h, ids, S, C.c_void_p(da[f].data_ptr()),
                                                  C.c_void_p(dt[f].data_ptr()), C.c_void_p(ts.cuda_stream)), "step")
    warm = min(3, F - 1)
    for f in range(warm):
        step(f)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ts)
    for f in range(warm, F):
        step(f)
    e1.record(ts)
    torch.cuda.synchronize()
    cache.close()
    return e0.elapsed_time(e1) / (F - warm), F - warm


Q4_SHAPES = [(6144, 2048), (2048, 2048), (16896, 2048), (2048, 8448), (8001, 2048)]  # (N rows, K)


def q4_sweep(torch, np, lib, stt_b200, device):
    """Configuration 5: isolated Q4_0 products, weights N(0, 0.02) quantised, activations N(0, 1)
    bf16.  M = 1 and 4 run the GEMV (bf16 input); M >= 16 the tensor-core GEMM (the bf16 activations
    converted to f16, exactly for these values).  After 3 warm-up calls, 20 back-to-back calls are
    captured in a CUDA graph and the graph is replayed 3 times between CUDA events: the device time
    per call, without the host's launch rate (a few microseconds per launch, as long as the smaller
    products themselves).  Returns [n, k, m, microseconds per call, path] rows."""
    out = []
    rng = np.random.default_rng(5)
    for n, k in Q4_SHAPES:
        raw = stt_b200.quantize_q4_0((rng.standard_normal(n * k) * 0.02).astype(np.float32))
        t = stt_b200.Q4Tensor.from_q4_bytes(raw, (n, k), device=device)
        for m in (1, 4, 16, 64, 256):
            x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
            dtype, xin = (1, x) if m < 16 else (2, x.to(torch.float16))
            y = torch.empty(m, n, dtype=torch.float32, device="cuda")

            def call(stream):
                rc = lib().stt_q4_matmul_device(t._h, xin.data_ptr(), dtype, m, y.data_ptr(), stream.cuda_stream)
                assert rc == 0, lib().stt_last_error().decode()
            side = torch.cuda.Stream()
            with torch.cuda.stream(side):
                for _ in range(3):
                    call(side)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                cs = torch.cuda.current_stream()
                for _ in range(20):
                    call(cs)
            torch.cuda.synchronize()
            ts = torch.cuda.current_stream()
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(ts)
            for _ in range(3):
                graph.replay()
            e1.record(ts)
            torch.cuda.synchronize()
            out.append([n, k, m, round(e0.elapsed_time(e1) / 60 * 1000.0, 2), "gemv" if m < 16 else "tcgen05"])
            del graph
        t.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5, help="timed steps (one step = the whole 250-frame job)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="only the headline workload")
    ap.add_argument("--frames", type=int, default=JOB_FRAMES,
                    help="frames per stream of the headline job; only a shorter profiling case sets it")
    ap.add_argument("--streams", type=int, default=JOB_STREAMS,
                    help="streams of the headline job; only a smaller profiling case sets it")
    ap.add_argument("--only", default="all", choices=["all", "job", "stream1", "streams64", "sweep", "frame"],
                    help="profiling cases: run one workload alone and print what it measured; 'frame' pre-rolls "
                         "--streams streams to --position with one persistent-kernel launch each, then times two "
                         "batched frames (few launches before them, for a profiler's launch list)")
    ap.add_argument("--position", type=int, default=129, help="position of the streams in the 'frame' case")
    ap.add_argument("--no-e2e", action="store_true", help="skip the per-call end-to-end timings (profiling cases)")
    ap.add_argument("--window", type=int, default=750,
                    help="sliding window of the model (K/V ring = window + 1 slots); only a profiling case "
                         "that must hold little device memory lowers it")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)

    import numpy as np
    import torch
    import stt_b200
    from stt_b200 import shard, synth
    from stt_b200._lib import lib, check

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        # the harness's only cross-rank traffic is a barrier and scalar reductions: gloo on CPU
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    def max_over_ranks(v):
        return shard.max_over_ranks(v, dist, "cpu")

    pk, pk_kind = peaks()
    ts = torch.cuda.current_stream()
    nthreads = max(1, len(os.sched_getaffinity(0)) // max(1, world))
    t0 = time.perf_counter()
    g = synth.synth_gguf(synth.SynthSpec(seed=SEED, n_threads=nthreads))
    t1 = time.perf_counter()
    cfg = stt_b200.SttConfig(text_start_token=0, sliding_window=args.window)   # initial text token 0
    # the first load of a process also pays its one-time set-up (kernel attributes, the pinned staging
    # ring, the copy threads); the rate reported is that of a second load, the first beside it
    model = stt_b200.SttModel.from_buffer(g.address, g.length, device=local, config=cfg)
    t2 = time.perf_counter()   # the load synchronises the device before it returns
    model.close()
    t3 = time.perf_counter()
    model = stt_b200.SttModel.from_buffer(g.address, g.length, device=local, config=cfg)
    t4 = time.perf_counter()
    load = {"gguf_bytes": g.length, "synth_s": round(t1 - t0, 3), "model_load_s": round(t4 - t3, 3),
            "model_load_gbs": round(g.length / (t4 - t3) / 1e9, 3),
            "first_load_in_process_s": round(t2 - t1, 3)}
    g.close()

    line = {}
    if args.only in ("all", "job"):
        # ---------------------------------------------------------------- headline: configuration 4
        total_streams, F = args.streams, args.frames
        blk = shard.stream_block(total_streams, world, rank)
        S = len(blk)
        cache = model.create_cache(S, "bf16")
        aud = np.stack([synth.audio_tokens(SEED, s, F) for s in blk], 1)   # [frame][stream][32]
        da = torch.from_numpy(aud.astype(np.int32)).cuda()
        dt = torch.empty(F, S, dtype=torch.int32, device="cuda")
        for _ in range(args.warmup):
            batched_job(model, cache, S, F, da, dt, lib, check, ts)
        barrier()
        with ClockSampler(local) as clk:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(ts)
            for _ in range(args.steps):
                batched_job(model, cache, S, F, da, dt, lib, check, ts)
            ev1.record(ts)
            torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        barrier()
        ms = max_over_ranks(ms)
        clocks = clk.summary()
        job_tokens = dt.cpu().numpy()     # [frame][stream] of the last step
        value = total_streams * F * args.steps / (ms / 1000.0)

        # tokens of the job's first streams against the oracle's (tests/golden/bench_tokens.json)
        token_check = None
        fx = os.path.join(REPO, "tests", "golden", "bench_tokens.json")
        if rank == 0 and os.path.exists(fx) and F == JOB_FRAMES:
            fxd = json.load(open(fx))
            ref = fxd["streams16_250"]
            ties = {(t[0], t[1]): t[2] for t in fxd["near_ties"]}
            k = min(len(ref), S)
            first = {}
            for s in range(k):
                d = np.nonzero(job_tokens[:, s] != np.array(ref[s]))[0]
                if d.size:
                    first[s] = int(d[0])
            token_check = {"streams_compared": k, "frames": F, "identical_streams": k - len(first),
                           # where a stream first differs, and the oracle's top-2 logit margin there
                           "first_difference": {str(s): [f, ties.get((s, f))] for s, f in first.items()}}

        # e2e: the same job through the public host-buffer call, one call per batched frame
        e2e_steps = 0 if args.no_e2e else min(args.steps, 3)
        audio_host = [np.ascontiguousarray(aud[f]) for f in range(F)]
        ids = list(range(S))
        if e2e_steps:
            for s in ids:                   # one untimed frame warms the host staging buffers
                cache.reset(s)
            cache.feed_frame(ids, audio_host[0])
        barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            for s in ids:
                cache.reset(s)
            for f in range(F):
                cache.feed_frame(ids, audio_host[f])
        e2e_s = time.perf_counter() - t0
        barrier()
        e2e_s = max_over_ranks(e2e_s)
        e2e = total_streams * F * e2e_steps / e2e_s if e2e_steps else None

        # the step's kernels and its dominant kernel, the tcgen05 GEMM, timed per launch
        nk = C.c_int()
        check(lib().stt_debug_graph_kernels(cache._h, S, C.byref(nk)), "graph_kernels")
        launches_per_step = S + F * (1 + nk.value)   # resets, then per frame the descriptor + the graph
        roofline = None
        if model.info.tensor_core_min_batch and S >= model.info.tensor_core_min_batch:
            us = (C.c_double * 5)()
            fl = (C.c_double * 5)()
            check(lib().stt_debug_time_products(cache._h, S, 20, us, fl), "time_products")
            per_step_us = 16 * (us[0] + us[1] + us[2] + us[3]) + us[4]
            per_step_flops = 16 * (fl[0] + fl[1] + fl[2] + fl[3]) + fl[4]
            achieved = per_step_flops / (per_step_us * 1e-6) / 1e12
            peak_t = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
            roofline = {"bound": "tensor", "kernel": "q4_tc_kernel (tcgen05 Q4_0 x f16 GEMM), the 65 products of a step",
                        "achieved": achieved, "peak": peak_t, "unit": "TFLOP/s", "frac": achieved / peak_t,
                        "peak_kind": f"{pk_kind} sustained bf16", "traffic": TC_TRAFFIC_LINEAR_IN_512,
                        "traffic_kernel": "one linear_in launch (16896 x 2048) at 512 rows",
                        "useful_flops_per_launch": per_step_flops / 65, "us_per_launch": per_step_us / 65,
                        "executed_mma_factor": 3,
                        "us_per_product": {"in_proj": us[0], "out_proj": us[1], "linear_in": us[2], "linear_out": us[3],
                                           "head": us[4]},
                        "gemm_share_of_step": per_step_us / (ms / args.steps / F * 1000.0)}
        # the same job with the two-product precision of the tensor-core layer products (activations
        # rounded to f16): a third less tensor work (stt_streams_set_product_precision)
        f16x2 = None
        if roofline is not None and not args.no_extras and args.only == "all":
            check(lib().stt_streams_set_product_precision(cache._h, 1), "set_product_precision")
            batched_job(model, cache, S, F, da, dt, lib, check, ts)
            barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(ts)
            for _ in range(2):
                batched_job(model, cache, S, F, da, dt, lib, check, ts)
            e1.record(ts)
            torch.cuda.synchronize()
            ms2 = max_over_ranks(e0.elapsed_time(e1))
            barrier()
            check(lib().stt_streams_set_product_precision(cache._h, 0), "set_product_precision")
            f16x2 = {"frames_per_s": total_streams * F * 2 / (ms2 / 1000.0), "ms_per_step": ms2 / 2,
                     "note": "two f16 products per weight (activation rounded to f16) instead of three"}
        step_bytes = algorithmic_bytes_batched([0] * S, 0, F)
        step_ms = ms / args.steps / F
        line = {
            "metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": job_config(world),
            "roofline": roofline,
            "e2e": {"value": e2e, "unit": "frames/s", "steps": e2e_steps,
                    "h2d_bytes_per_step": F * S * 32 * 4 + S * 32, "d2h_bytes_per_step": F * (S * 4 + 48)},
            "clocks": clocks,
            "gpu_launches": launches_per_step * args.steps,
            "batched_frame": {"ms": step_ms, "algorithmic_bytes": step_bytes,
                              "hbm_gbs": step_bytes / (step_ms / 1000.0) / 1e9,
                              "hbm_frac": step_bytes / (step_ms / 1000.0) / 1e9 / pk["hbm_gbs"],
                              "real_time_streams_per_gpu": S * 80.0 / step_ms},
            "tokens_vs_oracle": token_check,
            "products_f16x2": f16x2,
            "load": load,
        }
        cache.close()
        del da, dt

    if args.only == "frame":
        # one batched frame of S streams at position P, reached by one persistent-kernel launch per
        # stream (instead of P batched frames), then two batched frames
        S, P = args.streams, args.position
        cache = model.create_cache(S, "bf16")
        for s_ in range(S):
            pre = torch.from_numpy(synth.audio_tokens(SEED, s_, P).astype(np.int32)).cuda()
            tk = torch.empty(P, dtype=torch.int32, device="cuda")
            check(lib().stt_stream_feed_frames_device(cache._h, s_, P, C.c_void_p(pre.data_ptr()),
                                                      C.c_void_p(tk.data_ptr()), C.c_void_p(ts.cuda_stream)), "pre-roll")
        aud = np.stack([synth.audio_tokens(SEED, s_, 2, first_frame=P) for s_ in range(S)], 1)
        da = torch.from_numpy(aud.astype(np.int32)).cuda()
        dt = torch.empty(2, S, dtype=torch.int32, device="cuda")
        ids = (C.c_int32 * S)(*range(S))
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for f in range(2):
            if f == 1:
                e0.record(ts)
            check(lib().stt_streams_feed_frame_device(cache._h, ids, S, C.c_void_p(da[f].data_ptr()),
                                                      C.c_void_p(dt[f].data_ptr()), C.c_void_p(ts.cuda_stream)), "step")
        e1.record(ts)
        torch.cuda.synchronize()
        nk = C.c_int()
        check(lib().stt_debug_graph_kernels(cache._h, S, C.byref(nk)), "graph_kernels")
        line["frame"] = {"streams": S, "position": P, "ms": e0.elapsed_time(e1), "launches_before_second_frame":
                         3 * S + 1 + nk.value, "graph_kernels": nk.value}
        cache.close()
    extras = not args.no_extras
    if extras and args.only in ("all", "stream1"):
        # ------------------------------------------------------------ configuration 2: one stream
        c1 = model.create_cache(1, "bf16")
        st1 = stt_b200.SttStream(cfg, c1, 0)
        audio = synth.audio_tokens(SEED, rank, UTT_FRAMES)
        d_audio = torch.from_numpy(audio.astype(np.int32)).cuda()
        d_tokens = torch.empty(UTT_FRAMES, dtype=torch.int32, device="cuda")

        def utterance():
            check(lib().stt_stream_reset_async(c1._h, 0, 0, C.c_void_p(ts.cuda_stream)), "reset_async")
            check(lib().stt_stream_feed_frames_device(c1._h, 0, UTT_FRAMES, C.c_void_p(d_audio.data_ptr()),
                                                      C.c_void_p(d_tokens.data_ptr()), C.c_void_p(ts.cuda_stream)),
                  "feed_frames_device")
        n_utt = max(3, min(args.steps, 10))
        for _ in range(3):
            utterance()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ts)
        for _ in range(n_utt):
            utterance()
        e1.record(ts)
        torch.cuda.synchronize()
        ms1 = max_over_ranks(e0.elapsed_time(e1))
        toks1 = d_tokens.cpu().numpy()
        audio_host = [np.ascontiguousarray(a) for a in audio]
        e2e1 = float("nan")
        if not args.no_e2e:
            st1.reset()
            for f in range(3):
                st1.feed_frame(audio_host[f])
            barrier()
            t0 = time.perf_counter()
            for _ in range(2):
                st1.reset()
                for f in range(UTT_FRAMES):
                    st1.feed_frame(audio_host[f])
            e2e1 = max_over_ranks(time.perf_counter() - t0)
        algo = algorithmic_bytes_per_utterance(UTT_FRAMES)
        ach = algo / (ms1 / n_utt / 1000.0) / 1e9
        s1 = {"config": "1 stream x 750 frames per GPU (the persistent kernel)",
              "frames_per_s": world * n_utt * UTT_FRAMES / (ms1 / 1000.0), "ms_per_frame": ms1 / n_utt / UTT_FRAMES,
              "e2e_frames_per_s": world * 2 * UTT_FRAMES / e2e1,
              "vs_published_m2": (world * n_utt * UTT_FRAMES / (ms1 / 1000.0)) / world / PUBLISHED_FPS_750,
              "roofline": {"bound": "hbm", "kernel": "mega_kernel (one launch per utterance)", "achieved": ach,
                           "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": ach / pk["hbm_gbs"],
                           "algorithmic_bytes_per_step": algo, "traffic": MEGA_TRAFFIC_750}}
        fx = os.path.join(REPO, "tests", "golden", "bench_tokens.json")
        if rank == 0 and os.path.exists(fx):
            s1["tokens_identical_to_oracle"] = bool(np.array_equal(toks1, np.array(json.load(open(fx))["stream0_750"])))
        # where a late frame's time goes: every CTA's stamps of frame 740 (stt_debug_trace_frame)
        check(lib().stt_debug_trace_frame(c1._h, UTT_FRAMES - 10), "trace_frame")
        utterance()
        torch.cuda.synchronize()
        cap = 148 * 1024
        tb = (C.c_uint64 * cap)()
        n_ctas, n_slots = C.c_int(), C.c_int()
        if lib().stt_debug_get_trace_ctas(c1._h, tb, cap, C.byref(n_ctas), C.byref(n_slots)) == 0:
            s1["trace_frame_740"] = critical_path(list(tb[:n_ctas.value * n_slots.value]), n_ctas.value, n_slots.value, 16)
        check(lib().stt_debug_trace_frame(c1._h, -1), "trace_frame")
        c1.close()
        line["stream1"] = s1

    if extras and args.only in ("all", "streams64"):
        # ------------------------------------------------ configuration 3: 64 staggered streams
        offs = [round(i * 374 / 63) for i in range(64)]
        ms64, k64 = staggered(model, range(64 * rank, 64 * rank + 64), 375, offs, SEED, torch, np, lib, check, synth)
        barrier()
        ms64 = max_over_ranks(ms64)
        b64 = algorithmic_bytes_batched(offs, 375 - k64, 375)
        line["streams64"] = {"config": "64 streams per GPU, staggered offsets 0..374, 375 batched steps",
                             "frames_per_s": world * 64 * 1000.0 / ms64, "ms_per_step": ms64,
                             "real_time_streams_per_gpu": 64 * 80.0 / ms64,
                             "hbm_frac": b64 / (ms64 / 1000.0) / 1e9 / pk["hbm_gbs"]}
    if extras and args.only in ("all", "sweep"):
        if rank == 0:
            sweep = q4_sweep(torch, np, lib, stt_b200, local)
            gbs = {f"{n}x{k}": round(n * k // 32 * 18 / us / 1e3, 1) for n, k, m, us, _ in sweep if m == 1}
            line["q4_matmul"] = {"gemv_m1_weight_gbs": gbs, "gemv_m1_frac_of_hbm": max(gbs.values()) / pk["hbm_gbs"],
                                 "sweep_n_k_m_us_path": sweep}
        barrier()
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.only == "all":
        job = CpuJob()
        job.step()
        t0 = time.perf_counter()
        frames = sum(job.step() for _ in range(8))
        cpu_fps = frames / (time.perf_counter() - t0)
        line["cpu_baseline"] = {"value": cpu_fps, "unit": "frames/s", "cores": job.cores, "kind": "port",
                                "sample": job.sample() + ", 8 steps"}
    line["libraries"] = loaded_libraries()
    if rank == 0:
        # the per-configuration objects last: a reader of the end of the output sees them whole
        order = [k for k in line if k not in ("stream1", "streams64", "q4_matmul")] + \
                [k for k in ("q4_matmul", "stream1", "streams64") if k in line]
        print(json.dumps({k: line[k] for k in order}))
    model.close()
    if dist:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

#!/usr/bin/env python
"""Decode throughput of the STT-1B Q4 decode step on B200.

Workload (one bench step): one stream decodes a full 750-frame utterance (60 s of audio, the
whole sliding context) from position 0 with greedy token feedback: 16 layers, d_model 2048,
16 x 128 heads, FFN 8448, Q4_0 linear weights (627,351,552 bytes per frame), bf16 embeddings and
norms, bf16 KV.  Synthetic seeded weights N(0, 0.02) and seeded uniform audio tokens in
[0, 2048); initial text token 0.  With --gpus N each rank decodes its own stream on its own GPU
(independent streams, no collective): weak scaling.

  value  frames/s with audio tokens already in HBM, timed with CUDA events on the launch stream
  e2e    frames/s through the public per-frame call stt_stream_feed_frame (host audio in, host
         token out, one call per frame), host wall clock, max over ranks
  --impl reference  the CPU restatement of the reference decode step (oracle/) on the host cores
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

FRAMES = 750                     # frames per utterance (config: 750 frames, 60 s)
SEED = 0x5EED5EED
WEIGHT_BYTES = 627_351_552       # Q4_0 bytes of all linear layers, read once per frame
KV_BYTES_PER_TOKEN = 16 * 2 * 2048 * 2   # bf16 K+V of one cached position over 16 layers
EMB_BYTES = 33 * 2048 * 2        # 33 bf16 embedding rows per frame


# The reference's published 1-stream step time over a 750-frame (60 s) utterance: 52.5 ms per frame
# on an Apple M2 GPU through wgpu/Metal (BENCHMARKS.md:29 of stt-web).
PUBLISHED_FPS_750 = 1000.0 / 52.5

MEGA_TRAFFIC_750 = 508_142_132_480 + 2_654_166_784  # dram__bytes_read.sum + dram__bytes_write.sum, one launch


def algorithmic_bytes_per_utterance(frames=FRAMES, ring=751):
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


# Q4_0 weights of one step (16 layers + head), and the MMA work of a batched tensor-core step: three
# f16 MMAs per product (w_hi.x_hi + w_hi.x_lo + w_lo.x_hi) over the batch rows padded to the tile.
Q4_PARAMS = 16 * (6144 * 2048 + 2048 * 2048 + 16896 * 2048 + 2048 * 8448) + 8000 * 2048


def mma_flops_batched(S):
    nt = 16 if S <= 16 else 32 if S <= 32 else 64 if S <= 64 else 128 if S <= 128 else 256
    return 3 * 2 * ((S + nt - 1) // nt * nt) * Q4_PARAMS


def peaks():
    try:
        return json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json"))), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


TRACE_NAMES = {1: "frame_start", 11: "qkv_inputs", 12: "qkv_gemv", 13: "qkv_end", 21: "attention_inputs",
               22: "attention", 24: "attention_merge", 23: "attention_end", 31: "out_proj_inputs",
               32: "out_proj_gemv", 33: "out_proj_end", 41: "linear_in_inputs", 42: "linear_in_gemv",
               43: "linear_in_end", 51: "linear_out_inputs", 52: "linear_out_gemv", 53: "linear_out_end",
               61: "head_inputs", 62: "head_gemv", 63: "head_partial", 7: "argmax"}


def trace_breakdown(raw):
    """(tag, cycles) pairs of one traced frame of CTA 0, bracketed by (0, globaltimer ns) pairs ->
    microseconds spent reaching each kind of mark, plus the wait durations (tags >= 100: thread
    0's cycles + 1 in segment waits, 100 + kind, and flagged-word waits, 110 + kind)."""
    pairs = [(raw[i], raw[i + 1]) for i in range(0, len(raw) - 1, 2)]
    walls = [v for t, v in pairs if t == 0]
    marks = [(t, v) for t, v in pairs if 0 < t < 100]
    durs = [(t, v - 1) for t, v in pairs if t >= 100]
    frame_ns = walls[-1] - walls[0] if len(walls) >= 2 else None
    cycles = marks[-1][1] - marks[0][1]
    ns_per_cycle = frame_ns / cycles if frame_ns and cycles else 1.0 / 1.965
    out = {}
    for (t0, a), (t1, b) in zip(marks, marks[1:]):
        k = TRACE_NAMES.get(t1, str(t1))
        out[k] = out.get(k, 0.0) + (b - a) * ns_per_cycle / 1e3
    kinds = {1: "qkv", 2: "attention", 3: "out_proj", 4: "linear_in", 5: "linear_out", 6: "head"}
    waits = {}
    for t, v in durs:
        name = ("segment_wait_" if t < 110 else "input_wait_") + kinds.get(t % 10, str(t))
        waits[name] = waits.get(name, 0.0) + v * ns_per_cycle / 1e3
    return {"frame_us": frame_ns / 1e3 if frame_ns else None, "sm_ghz": 1.0 / ns_per_cycle,
            "trace_us": {k: round(v, 2) for k, v in out.items()},
            "cta0_waits_us": {k: round(v, 2) for k, v in sorted(waits.items())}}


LAYER_TAGS = [11, 12, 13, 21, 22, 24, 23, 31, 32, 33, 41, 42, 43, 51, 52, 53]
HEAD_TAGS = [61, 62, 63, 7]


def cta_breakdown(buf, n_ctas, n_slots, layers):
    """Per-CTA %globaltimer stamps of one frame -> how far the latest CTA moves at each kind of
    mark (critical path, us per frame) and how far it is ahead of the median CTA (lag)."""
    import numpy as np
    t = np.array(buf, dtype=np.int64).reshape(n_ctas, n_slots)
    starts = t[:, 0][t[:, 0] > 0]
    if starts.size == 0:
        return {}
    order = [(1 + 16 * l + i, tag) for l in range(layers) for i, tag in enumerate(LAYER_TAGS)]
    order += [(1 + 16 * layers + i, tag) for i, tag in enumerate(HEAD_TAGS)]
    prev = int(starts.max())
    crit, lag = {}, {}
    last = prev
    for slot, tag in order:
        v = t[:, slot][t[:, slot] > 0]
        if v.size == 0:
            continue
        mx = int(v.max())
        name = TRACE_NAMES.get(tag, str(tag))
        crit[name] = crit.get(name, 0.0) + (mx - prev) / 1e3
        lag[name] = lag.get(name, 0.0) + (mx - float(np.median(v))) / 1e3
        prev = mx
        last = mx
    return {"frame_us_all_ctas": (last - int(starts.min())) / 1e3,
            "critical_path_us": {k: round(v, 2) for k, v in crit.items()},
            "lag_behind_median_us": {k: round(v, 2) for k, v in lag.items()}}


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


def cpu_reference(frames_budget_s, warmup, steps, threads=None):
    """Times the oracle (CPU restatement of the reference step, reference f32 precision)."""
    import numpy as np
    import stt_b200
    from oracle import oracle as O
    if threads:
        O.set_threads(threads)
    g = stt_b200.synth_gguf(stt_b200.SynthSpec(seed=SEED))
    om = O.OracleModel(g.array, text_start_token=0)
    s = om.stream(0)
    audio = stt_b200.audio_tokens(SEED, 0, FRAMES)
    for f in range(min(warmup, 3)):
        s.feed_frame(audio[f])
    done, t0 = 0, time.perf_counter()
    f = min(warmup, 3)
    target = min(steps * FRAMES, FRAMES - f)
    while done < target:
        s.feed_frame(audio[f])
        f += 1
        done += 1
        if time.perf_counter() - t0 > frames_budget_s:
            break
    dt = time.perf_counter() - t0
    return done / dt, done, O.get_threads()


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    fps, n, cores = cpu_reference(120.0, args.warmup, args.steps)
    sample = f"{n} consecutive frames (positions 3..{3 + n - 1}) of the 750-frame utterance, f32 reference precision"
    line = {
        "impl": "reference", "metric": "decode frames/s per GPU (1 stream, 750-frame utterance)",
        "value": fps, "unit": "frames/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": FRAMES * 1000.0 / fps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "1 stream x 750 frames (config 2), STT-1B Q4_0, 16 layers d2048"},
        "cpu_baseline": {"value": fps, "unit": "frames/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": fps, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def multi_stream(model, stream_ids, F, offsets, seed, torch, np, lib, check, stt_b200):
    """Config 3 / 4 workload on this GPU: the S = len(stream_ids) streams of those global ids, the s-th
    pre-rolled alone to offsets[s] frames, then F batched steps of all S streams (one frame each),
    device-timed.  A stream's audio tokens follow from (seed, global id), so it decodes the same
    frames whichever rank holds it.  Returns ms per step and the number of timed steps (the last
    F - warm of the F)."""
    S = len(stream_ids)
    cache = model.create_cache(S, "bf16")
    ts = torch.cuda.current_stream()
    for s_ in range(S):
        if offsets[s_]:
            pre = stt_b200.audio_tokens(seed, stream_ids[s_], offsets[s_])
            a = torch.from_numpy(pre.astype(np.int32)).cuda()
            tk = torch.empty(offsets[s_], dtype=torch.int32, device="cuda")
            check(lib().stt_stream_feed_frames_device(cache._h, s_, offsets[s_], C.c_void_p(a.data_ptr()),
                                                      C.c_void_p(tk.data_ptr()), C.c_void_p(ts.cuda_stream)), "pre-roll")
    aud = np.stack([stt_b200.audio_tokens(seed, stream_ids[s_], F, first_frame=offsets[s_]) for s_ in range(S)], 1)
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
    """Config 5: isolated Q4_0 products, weights N(0, 0.02) quantised, activations N(0, 1) bf16.
    M = 1 and 4 run the GEMV (bf16 input); M >= 16 the tensor-core GEMM (the bf16 activations
    converted to f16, exactly for these values).  Device-timed, 20 calls after 3 warm-up calls."""
    out = []
    rng = np.random.default_rng(5)
    ts = torch.cuda.current_stream()
    for n, k in Q4_SHAPES:
        raw = stt_b200.quantize_q4_0((rng.standard_normal(n * k) * 0.02).astype(np.float32))
        t = stt_b200.Q4Tensor.from_q4_bytes(raw, (n, k), device=device)
        for m in (1, 4, 16, 64, 256):
            x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
            dtype, xin = (1, x) if m < 16 else (2, x.to(torch.float16))
            y = torch.empty(m, n, dtype=torch.float32, device="cuda")

            def call():
                rc = lib().stt_q4_matmul_device(t._h, xin.data_ptr(), dtype, m, y.data_ptr(), ts.cuda_stream)
                assert rc == 0, lib().stt_last_error().decode()
            for _ in range(3):
                call()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(ts)
            for _ in range(20):
                call()
            e1.record(ts)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / 20 * 1000.0
            out.append({"n": n, "k": k, "m": m, "us": round(us, 2), "path": "gemv" if m < 16 else "tcgen05",
                        "weight_gbs": round(n * k // 32 * 18 / us / 1e3, 1),
                        "tflops": round(2.0 * n * k * m / us / 1e6, 2)})
        t.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10, help="timed utterances of 750 frames")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--frames", type=int, default=FRAMES,
                    help="frames per utterance; only a shorter profiling case sets it (default 750)")
    ap.add_argument("--no-multi", action="store_true", help="skip the 64- and 512-stream and matmul-sweep lines")
    ap.add_argument("--batched", type=int, default=0,
                    help="profiling case: only S streams x --frames batched steps from position 0, one JSON line")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)

    import numpy as np
    import torch
    import stt_b200
    from stt_b200 import shard
    from stt_b200._lib import lib, check

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    nframes = args.frames
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        return shard.max_over_ranks(v, dist, "cuda")

    nthreads = max(1, (os.cpu_count() or 8) // max(1, world))
    t0 = time.perf_counter()
    g = stt_b200.synth_gguf(stt_b200.SynthSpec(seed=SEED, n_threads=nthreads))
    t1 = time.perf_counter()
    cfg = stt_b200.SttConfig(text_start_token=0)   # initial text token 0 (benchmark config)
    model = stt_b200.SttModel.from_buffer(g.address, g.length, device=local, config=cfg)
    t2 = time.perf_counter()   # the load synchronises the device before it returns
    load = {"gguf_bytes": g.length, "synth_s": t1 - t0, "model_load_s": t2 - t1,
            "model_load_gbs": g.length / (t2 - t1) / 1e9}
    g.close()
    if args.batched:
        ms_b, k_b = multi_stream(model, range(args.batched), nframes, [0] * args.batched, SEED, torch, np, lib,
                                 check, stt_b200)
        if rank == 0:
            print(json.dumps({"batched_streams": args.batched, "frames": nframes, "timed_steps": k_b,
                              "ms_per_step": ms_b, "frames_per_s": args.batched * 1000.0 / ms_b}))
        model.close()
        return 0
    cache = model.create_cache(1, "bf16")
    stream = stt_b200.SttStream(cfg, cache, 0)
    audio = stt_b200.audio_tokens(SEED, rank, nframes)
    d_audio = torch.from_numpy(audio.astype(np.int32)).cuda()
    d_tokens = torch.empty(nframes, dtype=torch.int32, device="cuda")
    ts = torch.cuda.current_stream()

    def utterance_device():
        check(lib().stt_stream_reset_async(cache._h, 0, 0, C.c_void_p(ts.cuda_stream)), "reset_async")
        check(lib().stt_stream_feed_frames_device(cache._h, 0, nframes, C.c_void_p(d_audio.data_ptr()),
                                                  C.c_void_p(d_tokens.data_ptr()), C.c_void_p(ts.cuda_stream)),
              "feed_frames_device")

    # ---- value: device-resident inputs
    for _ in range(args.warmup):
        utterance_device()
    torch.cuda.synchronize()
    barrier()
    with ClockSampler(local) as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(ts)
        for _ in range(args.steps):
            utterance_device()
        ev1.record(ts)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    barrier()
    ms = max_over_ranks(ms)
    clocks = clk.summary()
    dev_tokens = d_tokens.cpu().numpy()
    value = world * args.steps * nframes / (ms / 1000.0)

    # ---- e2e: the public per-frame call with host buffers
    audio_host = [np.ascontiguousarray(a) for a in audio]
    stream.reset()
    for f in range(3):
        stream.feed_frame(audio_host[f])
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        stream.reset()
        for f in range(nframes):
            stream.feed_frame(audio_host[f])
    e2e_s = time.perf_counter() - t0
    barrier()
    e2e_s = max_over_ranks(e2e_s)
    e2e = world * args.steps * nframes / e2e_s

    # ---- diagnostics: grid-barrier latency and a per-phase breakdown of one late frame
    diag = {}
    ns = C.c_double()
    if lib().stt_debug_barrier_ns(local, 2000, 0, C.byref(ns)) == 0:
        diag["grid_barrier_ns"] = ns.value
    if lib().stt_debug_barrier_ns(local, 2000, 1, C.byref(ns)) == 0:
        diag["grid_barrier_flag_ns"] = ns.value
    lib().stt_debug_trace_frame(cache._h, nframes - 10)
    utterance_device()
    torch.cuda.synchronize()
    buf = (C.c_uint64 * 1024)()
    nt = C.c_int()
    if lib().stt_debug_get_trace(cache._h, buf, 1024, C.byref(nt)) == 0 and nt.value > 4:
        diag.update(trace_breakdown([buf[i] for i in range(nt.value)]))
        diag["traced_frame"] = nframes - 10
    cap = 148 * 1024
    tb = (C.c_uint64 * cap)()
    nc, ns_ = C.c_int(), C.c_int()
    if lib().stt_debug_get_trace_ctas(cache._h, tb, cap, C.byref(nc), C.byref(ns_)) == 0:
        diag.update(cta_breakdown(list(tb[:nc.value * ns_.value]), nc.value, ns_.value, 16))
    lib().stt_debug_trace_frame(cache._h, -1)

    # ---- roofline of the decode step (every kernel of a frame, device-timed above)
    pk, pk_kind = peaks()
    algo = algorithmic_bytes_per_utterance(nframes)
    achieved = algo / (ms / args.steps / 1000.0) / 1e9
    line = {
        "metric": "decode frames/s per GPU (1 stream, 750-frame utterance)",
        "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "ms_per_frame": ms / args.steps / nframes,
        "higher_is_better": True, "scaling": "weak",
        # against the published single-stream rate (other hardware), at the full 750 frames only
        "vs_baseline": value / PUBLISHED_FPS_750 if nframes == FRAMES else None,
        "vs_baseline_source": "stt-web BENCHMARKS.md:29: 52.5 ms/frame, 1 stream x 750 frames, Apple M2 wgpu/Metal",
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"1 stream x {nframes} frames per GPU, STT-1B Q4_0, 16 layers d2048, bf16 KV",
                   "l2": "inputs larger than L2: 627 MB of Q4 weights streamed per frame",
                   "parallelism": f"{world} independent streams, one per GPU"},
        "roofline": {"bound": "hbm", "kernel": "decode step (all kernels of one frame)", "achieved": achieved,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "peak_kind": pk_kind, "algorithmic_bytes_per_step": algo,
                     # DRAM read + write bytes of one 750-frame launch, from the ncu capture in
                     # profiles/mega_kernel_dram_750frames.txt (not measured for other frame counts)
                     "traffic": MEGA_TRAFFIC_750 if nframes == FRAMES else None},
        "e2e": {"value": e2e, "unit": "frames/s", "h2d_bytes_per_step": nframes * 32 * 4,
                "d2h_bytes_per_step": nframes * (4 + 32)},
        "clocks": clocks,
        # this rank's model load from a host buffer (parse, upload, repack), host wall clock
        "load": load,
        # our kernels per step: stream reset, step descriptor, audio-embedding sums, persistent kernel
        "gpu_launches": 4 * args.steps,
        "diagnostics": diag,
        "tokens_checksum": int(np.int64(dev_tokens.astype(np.int64).sum())),
    }
    if not args.no_multi:
        # config 3: 64 streams per GPU at staggered offsets 0..374, 375 batched steps
        offs = [round(i * 374 / 63) for i in range(64)]
        ms64, k64 = multi_stream(model, range(64 * rank, 64 * rank + 64), 375, offs, SEED, torch, np, lib, check,
                                 stt_b200)
        barrier()
        ms64 = max_over_ranks(ms64)
        b64 = algorithmic_bytes_batched(offs, 375 - k64, 375)
        line["streams64"] = {"frames_per_s": world * 64 * 1000.0 / ms64, "ms_per_step": ms64, "timed_steps": k64,
                             "real_time_streams_per_gpu_at_this_batch": 64 * 80.0 / ms64,
                             "roofline": {"bound": "hbm", "algorithmic_bytes_per_step": b64,
                                          "achieved": b64 / (ms64 / 1000.0) / 1e9, "peak": pk["hbm_gbs"],
                                          "unit": "GB/s", "frac": b64 / (ms64 / 1000.0) / 1e9 / pk["hbm_gbs"]},
                             "tensor": {"mma_flops_per_step": mma_flops_batched(64),
                                        "achieved_tflops_over_step": mma_flops_batched(64) / (ms64 / 1000.0) / 1e12,
                                        "peak": pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")),
                                        "peak_kind": "sustained bf16 (a seconds-long loop)", "unit": "TFLOP/s"},
                             "config": "64 streams per GPU, staggered offsets 0..374, 375 frames each, bf16 KV, "
                                       "layer products on tcgen05 (M = 64)"}
        # config 4: 512 streams split into contiguous blocks over the GPUs, 250 frames each
        blk = shard.stream_block(512, world, rank)
        per = len(blk)
        ms512, k512 = multi_stream(model, blk, 250, [0] * per, SEED, torch, np, lib, check, stt_b200)
        barrier()
        ms512 = max_over_ranks(ms512)
        total512 = shard.sum_over_ranks(per, dist, "cuda")
        b512 = algorithmic_bytes_batched([0] * per, 250 - k512, 250)
        line["streams512"] = {"frames_per_s": total512 * 1000.0 / ms512, "ms_per_step": ms512,
                              "timed_steps": k512, "config": f"{per} streams per GPU x {world} GPUs, 250 frames",
                              "roofline": {"bound": "hbm", "algorithmic_bytes_per_step": b512,
                                           "achieved": b512 / (ms512 / 1000.0) / 1e9, "peak": pk["hbm_gbs"],
                                           "unit": "GB/s", "frac": b512 / (ms512 / 1000.0) / 1e9 / pk["hbm_gbs"]},
                              "tensor": {"mma_flops_per_step": mma_flops_batched(per),
                                         "achieved_tflops_over_step": mma_flops_batched(per) / (ms512 / 1000.0) / 1e12,
                                         "peak": pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")),
                                         "peak_kind": "sustained bf16 (a seconds-long loop)", "unit": "TFLOP/s"}}
        if rank == 0:
            sweep = q4_sweep(torch, np, lib, stt_b200, local)
            m1 = [r for r in sweep if r["m"] == 1]
            line["q4_matmul"] = {"gemv_m1_weight_gbs": {f"{r['n']}x{r['k']}": r["weight_gbs"] for r in m1},
                                 "gemv_m1_frac_of_hbm": max(r["weight_gbs"] for r in m1) / pk["hbm_gbs"],
                                 "sweep": sweep}
        barrier()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        fps, n, cores = cpu_reference(20.0, 3, 1)
        line["cpu_baseline"] = {"value": fps, "unit": "frames/s", "cores": cores, "kind": "port",
                                "sample": f"{n} frames of the same utterance (positions 3..{2 + n}), oracle f32"}
    if rank == 0:
        print(json.dumps(line))
    cache.close()
    model.close()
    if dist:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

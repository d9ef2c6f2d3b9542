"""Generates tests/golden/bench_tokens.json: the oracle's tokens for the benchmark's own inputs.

    python tests/golden/make_bench_tokens.py

The benchmark decodes the full-size synthetic STT-1B checkpoint (SynthSpec() defaults, seed
0x5EED5EED) with the initial text token 0, bf16 K/V and the feed_frame loop (text delay 6,
limit-cycle rule), each stream s reading the seeded audio tokens audio_tokens(seed, s, ...).
This script runs the CPU oracle (oracle/, the restatement of the reference step, with its K/V
rounded to bf16 as the library stores them) on those inputs:

  stream0_750    the 750 feed_frame results of stream 0 (the 1-stream, 750-frame workload)
  streams16_250  the first 250 results of streams 0..15 (the first streams of the 512-stream,
                 250-frame workload; streams are independent, so a batch of any size must give
                 each of them these tokens)
  near_ties      every (stream, frame, top-2 logit margin) with a margin below 5e-2, so that a
                 mismatch can be told apart from a genuine near-tie

and tests/golden/bench_logits.npz: stream 0's logits at frames 6, 100, 249, 400, 700 and 749.

None (a frame inside the text delay) is written as -1.  Takes a few minutes on 8 cores.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
for p in (os.path.join(REPO, "stt-web_b200"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

SEED = 0x5EED5EED
TIE = 5e-2
LOGIT_FRAMES = (6, 100, 249, 400, 700, 749)


def margin(lg):
    s = np.sort(lg)
    return float(s[-1] - s[-2])


def main():
    from oracle import oracle as O
    from stt_b200 import synth

    O.set_threads(len(os.sched_getaffinity(0)))
    g = synth.synth_gguf(synth.SynthSpec(seed=SEED))
    om = O.OracleModel(g.array, text_start_token=0)
    n = 16
    streams = [om.stream(O.KV_BF16) for _ in range(n)]
    audio = np.stack([synth.audio_tokens(SEED, s, 750) for s in range(n)], 1)  # [frame][stream][32]
    toks = [[] for _ in range(n)]
    ties = []
    logits = {}
    for f in range(250):
        t, lg = O.feed_frame_batch(streams, audio[f], want_logits=True)
        if f in LOGIT_FRAMES:
            logits[f] = lg[0].copy()
        for s in range(n):
            toks[s].append(-1 if t[s] is None else t[s])
            m = margin(lg[s])
            if m < TIE:
                ties.append([s, f, m])
        if f % 50 == 0:
            print("frame", f, flush=True)
    s0 = list(toks[0])
    for f in range(250, 750):
        t, lg = streams[0].feed_frame_logits(audio[f, 0])
        s0.append(-1 if t is None else t)
        if f in LOGIT_FRAMES:
            logits[f] = lg.copy()
        m = margin(lg)
        if m < TIE:
            ties.append([0, f, m])
        if f % 100 == 0:
            print("frame", f, flush=True)
    out = {"seed": SEED, "text_start_token": 0, "kv": "bf16", "oracle_flags": "KV_BF16",
           "stream0_750": s0, "streams16_250": toks, "near_ties": ties}
    with open(os.path.join(HERE, "bench_tokens.json"), "w") as fh:
        json.dump(out, fh, separators=(",", ":"))
    np.savez_compressed(os.path.join(HERE, "bench_logits.npz"), frames=np.array(LOGIT_FRAMES),
                        logits=np.stack([logits[f] for f in LOGIT_FRAMES]))
    print("written; near ties:", len(ties))


if __name__ == "__main__":
    main()

"""The multi-GPU host logic on CPU: two `gloo` ranks on 127.0.0.1.

A job of independent streams spreads over ranks by contiguous blocks of global stream ids
(stt_b200.shard.stream_block), each rank decoding its block on its own weight replica; streams
share no state (crates/stt-wasm/src/model.rs:263-296), so the union of the ranks' tokens must
equal the unsharded job's.  The decoding here is the oracle's (CPU): what is under test is the
partition, the per-stream inputs named by global id, and the rank reductions that the bench's
timing uses (slowest rank, units summed), including a rank that leaves before a reduction.
"""
import datetime
import json
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from stt_b200 import shard

SEED = 0x5EED5EED


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, seconds=30):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=seconds))
    return dist


def _stream_audio(meta, sid, frames):
    import stt_b200
    # the bench's per-stream inputs: seeded by the global stream id, folded into the tiny model's vocabulary
    return stt_b200.audio_tokens(SEED, sid, frames, num_codebooks=meta["codebooks"]) % meta["audio_vocab"]


def _decode(gguf, meta, sids, frames):
    from oracle import oracle as O
    m = O.OracleModel(gguf, num_layers=meta["num_layers"], num_heads=meta["heads"],
                      num_codebooks=meta["codebooks"], text_start_token=meta["text_vocab"] - 1)
    out = {}
    for sid in sids:
        s = m.stream()
        out[sid] = [s.feed_frame(a) for a in _stream_audio(meta, sid, frames)]
    return out


def _sharded_job(rank, world, port, gguf, meta, total, frames, out_path):
    dist = _init(rank, world, port)
    blk = shard.stream_block(total, world, rank)
    toks = _decode(gguf, meta, blk, frames)
    gathered = [None] * world
    dist.all_gather_object(gathered, {"block": [blk.start, blk.stop], "tokens": toks})
    res = {
        "gathered": gathered,
        "max": shard.max_over_ranks(1.5 * (rank + 1), dist),
        "sum": shard.sum_over_ranks(len(blk), dist),
        # rank r reports len(blk) * frames units in (r + 1) seconds: the job's rate is bounded by the slowest
        "rate": shard.job_rate(len(blk) * frames, float(rank + 1), dist),
    }
    if rank == 0:
        with open(out_path, "w") as f:
            json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


def test_stream_blocks_cover_every_stream_once():
    for total in (0, 1, 5, 64, 511, 512, 513):
        for world in (1, 2, 3, 4, 8):
            blocks = [shard.stream_block(total, world, r) for r in range(world)]
            ids = [i for b in blocks for i in b]
            assert ids == list(range(total))
            sizes = [len(b) for b in blocks]
            assert max(sizes) - min(sizes) <= 1 and sizes == sorted(sizes, reverse=True)
    assert shard.stream_block(512, 8, 3) == range(192, 256)
    with pytest.raises(ValueError):
        shard.stream_block(8, 2, 2)
    with pytest.raises(ValueError):
        shard.stream_block(-1, 1, 0)


def test_reductions_without_a_process_group():
    assert shard.max_over_ranks(2.5) == 2.5
    assert shard.sum_over_ranks(7) == 7.0
    assert shard.job_rate(100, 2.0) == 50.0
    with pytest.raises(ValueError):
        shard.job_rate(1, 0.0)


def test_two_gloo_ranks_decode_the_unsharded_job(tiny_ref_gguf, tiny_meta, tmp_path):
    total, frames, world = 5, 10, 2
    out = str(tmp_path / "rank0.json")
    mp.start_processes(_sharded_job, args=(world, _free_port(), tiny_ref_gguf, tiny_meta, total, frames, out),
                       nprocs=world, join=True, start_method="spawn")
    res = json.load(open(out))
    blocks = [tuple(g["block"]) for g in res["gathered"]]
    assert blocks == [(0, 3), (3, 5)]
    sharded = {int(k): v for g in res["gathered"] for k, v in g["tokens"].items()}
    assert sorted(sharded) == list(range(total))
    whole = _decode(tiny_ref_gguf, tiny_meta, range(total), frames)
    assert sharded == whole
    # the streams differ from one another, so the comparison above is not vacuous
    assert len({tuple(_stream_audio(tiny_meta, s, frames).ravel()) for s in range(total)}) == total
    assert res["max"] == 3.0
    assert res["sum"] == total
    assert res["rate"] == pytest.approx(total * frames / 2.0)


def _rank_leaves(rank, world, port, out_path):
    dist = _init(rank, world, port, seconds=20)
    dist.barrier()
    if rank == 1:
        # leaves between steps, with nothing in flight; its process exits without a further collective
        os._exit(0)
    try:
        shard.max_over_ranks(1.0, dist)
        outcome = "returned"
    except Exception as e:  # noqa: BLE001 - any transport or timeout error is the expected outcome
        outcome = "raised: " + type(e).__name__
    with open(out_path, "w") as f:
        f.write(outcome)
    os._exit(0)


def test_a_departed_rank_makes_the_reduction_raise(tmp_path):
    out = str(tmp_path / "rank0.txt")
    ctx = mp.start_processes(_rank_leaves, args=(2, _free_port(), out), nprocs=2, join=False, start_method="spawn")
    deadline = datetime.datetime.now() + datetime.timedelta(seconds=90)
    while not ctx.join(timeout=5):
        assert datetime.datetime.now() < deadline, "rank 0 waited for the departed rank past the group timeout"
    assert open(out).read().startswith("raised")

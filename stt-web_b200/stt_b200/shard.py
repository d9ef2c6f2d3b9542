"""Independent streams spread over GPUs, one process per GPU.

Streams share nothing but the read-only weights: every stream owns its KV cache and its token
state (``SttModel::create_cache`` and ``LayerCaches``, crates/stt-wasm/src/model.rs:263-296,
728-738; ``SttStream`` state, crates/stt-wasm/src/stream.rs:19-60).  A job of S streams on G GPUs
is therefore G independent jobs: rank r decodes a contiguous block of stream ids on its own
weight replica, and no activation, cache or token crosses GPUs.  The only cross-rank values are
scalars of the bookkeeping: the slowest rank's time bounds the job.

A stream's inputs are named by its global id, so a stream decodes the same frames whatever the
number of ranks, and a sharded job produces exactly the tokens of the unsharded one.
"""
from __future__ import annotations


def stream_block(total: int, world: int, rank: int) -> range:
    """Contiguous block of global stream ids that ``rank`` decodes when ``total`` streams are
    spread over ``world`` ranks.  Block sizes differ by at most one; the first ``total % world``
    ranks take one stream more.  Raises ValueError for a negative total or a rank outside the
    world."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError(f"stream_block: total={total}, world={world}, rank={rank}")
    base, extra = divmod(total, world)
    first = rank * base + min(rank, extra)
    return range(first, first + base + (1 if rank < extra else 0))


def max_over_ranks(value: float, dist=None, device="cpu") -> float:
    """The largest ``value`` over all ranks of the default process group (``value`` itself
    without one).  Every rank must call it at the same point; a rank that has left makes the
    others raise once the group's timeout or the transport notices, instead of waiting for good."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, dist=None, device="cpu") -> float:
    """The sum of ``value`` over all ranks (``value`` itself without a process group)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def job_rate(units: float, seconds: float, dist=None, device="cpu") -> float:
    """Whole-job throughput: the units every rank processed, summed, divided by the slowest
    rank's time.  ``units`` and ``seconds`` are this rank's own."""
    total = sum_over_ranks(units, dist, device)
    slowest = max_over_ranks(seconds, dist, device)
    if slowest <= 0.0:
        raise ValueError("job_rate: the slowest rank reported no time")
    return total / slowest

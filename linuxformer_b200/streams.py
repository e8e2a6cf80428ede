"""Independent decode streams over several GPUs: one process per GPU, one machine per process.

The chip decode does not shard inside a stream (every token depends on the previous one through
the whole stack), so N GPUs run N independent machines: rank r decodes its own stream from its
own state, with no collective on the decode path. The only exchange is the host-side timing
reduction of a benchmark (the slowest rank's device time). Works with the ``nccl`` backend on
GPUs and ``gloo`` on CPU (the multi-rank tests).
"""

from __future__ import annotations

import os


def rank_env() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment (1 process when unset)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def stream_seed(base: int, rank: int) -> int:
    """The state seed of rank ``rank``'s machine: every rank a different stream."""
    return base + rank


def slowest(values, device=None) -> list[float]:
    """Element-wise maximum of ``values`` over all ranks (the identity with one process)."""
    import torch
    import torch.distributed as dist

    vals = [float(v) for v in values]
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return vals
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.cpu()]


def job_rate(units_per_rank: float, world: int, slowest_seconds: float) -> float:
    """Whole-job throughput: the units every rank processed over the slowest rank's time."""
    if slowest_seconds <= 0:
        raise ValueError("a non-positive time")
    return units_per_rank * world / slowest_seconds


def shard(n_streams: int, rank: int, world: int) -> list[int]:
    """The streams rank ``rank`` runs when ``n_streams`` independent machines are split evenly
    over ``world`` GPUs: a contiguous block of n_streams / world (config 4: 64 streams over
    1/2/4/8 GPUs)."""
    if world < 1 or not 0 <= rank < world or n_streams % world:
        raise ValueError(f"{n_streams} streams do not split evenly over {world} ranks")
    k = n_streams // world
    return list(range(rank * k, (rank + 1) * k))


def gather_digests(mine: dict[int, str], device=None) -> dict[int, str]:
    """Every rank's {stream: digest}, merged on every rank (a host-side object gather after the
    timed region; the decode path itself exchanges nothing)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return dict(mine)
    parts = [None] * dist.get_world_size()
    dist.all_gather_object(parts, mine)
    out: dict[int, str] = {}
    for p in parts:
        out.update(p)
    return out

"""Independent streams sharded across the GPUs of one box (one process per GPU).

Decode streams never exchange data, so the multi-GPU path is weak scaling by
stream with no collective on the data path: GPU g holds a full weight replica
and decodes global streams [g * per_gpu, (g + 1) * per_gpu) (the 512 streams
of the 8-GPU configuration are 64 per GPU). torch.distributed serves only the
host side -- a barrier around the timed region and the max over ranks of the
device times -- with NCCL on GPUs and gloo on CPU.
"""

from __future__ import annotations

import numpy as np


def shard(total: int, world: int, rank: int) -> range:
    """Global stream ids of `rank`: contiguous, balanced, disjoint, covering."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return range(total * rank // world, total * (rank + 1) // world)


def prefix_lengths(lo: int, hi: int, seed: int, total: int) -> list[int]:
    """Audio-prefix rows of `total` global streams, uniform in [lo, hi] from
    one generator per workload; a draw of more streams extends a draw of fewer
    (numpy draws bounded integers in sequence), so stream g's length does not
    depend on the number of GPUs."""
    return [int(x) for x in np.random.default_rng([seed, 3]).integers(lo, hi + 1, size=total)]


def max_over_ranks(value: float) -> float:
    """The maximum of `value` over all ranks of the default process group (the
    slowest rank's time); `value` itself without one."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def aggregate_rate(units_per_rank: int, world: int, seconds: float) -> float:
    """Whole-job throughput: the units every rank processed over the slowest
    rank's time."""
    return units_per_rank * world / seconds

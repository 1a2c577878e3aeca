"""Batch sharding across the GPUs of one node.

Every operation on the forecast-guided sparse-attention path is per sequence
(compressor, selector, attention, prefetch: model/forecast.py and
model/attention/*.py never mix batch rows), so requests shard by batch row with
no collective on the hot path.  One process per GPU; the only collectives are
the host-side barrier and timing reductions used by the benchmark.
"""

from __future__ import annotations

from typing import Tuple


def batch_shard(global_batch: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [start, stop) rows of ``global_batch`` owned by ``rank``;
    the first ``global_batch % world`` ranks take one extra row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if global_batch < 0:
        raise ValueError(f"negative batch {global_batch}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def max_over_ranks(x: float, device=None) -> float:
    """Maximum of a per-rank scalar over the default process group (the
    slowest rank sets a step's time); identity without a process group."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, device=None) -> float:
    """Sum of a per-rank scalar (e.g. tokens processed) over the default
    process group; identity without a process group."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())

"""Row (token) partitioning across GPUs, and the timing reduction.

Every op on the path is row-independent, so multi-GPU work needs no collective
on the data path: each rank owns a contiguous block of rows (tokens) and its own
sequences' cache slots. torch.distributed is used only as plumbing — a barrier
around the timed region and a MAX reduction of the measured times.
"""
from __future__ import annotations

from typing import Sequence


def weak_rows(rank: int, world: int, rows_per_rank: int) -> range:
    """Weak scaling: rank r owns global rows [r * R, (r + 1) * R) of an N * R job."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside [0, {world})")
    if rows_per_rank < 0:
        raise ValueError("rows_per_rank must be >= 0")
    return range(rank * rows_per_rank, (rank + 1) * rows_per_rank)


def strong_rows(rank: int, world: int, total_rows: int) -> range:
    """Strong scaling: total_rows split into contiguous blocks of ceil(total/world)
    rows (the last blocks may be shorter or empty)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside [0, {world})")
    block = -(-total_rows // world)
    start = min(total_rows, rank * block)
    return range(start, min(total_rows, start + block))


def max_over_ranks(values: Sequence[float], device=None) -> list:
    """Element-wise MAX of `values` over all ranks (identity without a process group)."""
    import torch
    import torch.distributed as dist

    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()

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


def local_shape(shape, rank: int, world: int, scaling: str = "strong"):
    """This rank's share of a layer-step workload: (shape with this rank's rows
    and sequences, global row range).

    strong: the workload's rows split into contiguous blocks of ceil(R/world);
            the cache holds only the sequences those rows touch (a sequence cut
            between ranks keeps its positions: each rank writes its own slots).
    weak:   every rank owns a whole copy of the workload's rows (an N x R job).
    """
    import dataclasses

    if scaling == "weak":
        rows = weak_rows(rank, world, shape.rows)
        return shape, rows
    if scaling != "strong":
        raise ValueError(f"scaling must be 'strong' or 'weak', got {scaling!r}")
    rows = strong_rows(rank, world, shape.rows)
    n = len(rows)
    if shape.positions == "tiled":
        seqs = (-(-rows.stop // shape.max_seq) - rows.start // shape.max_seq) if n else 1
    else:
        seqs = max(1, min(shape.num_seqs, n))
    return dataclasses.replace(shape, rows=n, num_seqs=max(1, seqs)), rows


def max_over_ranks(values: Sequence[float], device=None) -> list:
    """Element-wise MAX of `values` over all ranks (identity without a process group)."""
    import torch
    import torch.distributed as dist

    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()

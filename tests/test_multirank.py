"""The multi-GPU host logic on CPU: two `gloo` ranks on 127.0.0.1.

* Row partitioning: weak and strong splits are disjoint and cover the job;
  each rank's token layout (positions, sequence ids) is a valid shard.
* The timing reduction returns the maximum over ranks.
* Failure detection without a GPU: a rank that dies before the barrier makes the
  survivor's barrier fail within the process-group timeout instead of hanging.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from baremetalinferenceengine_b200 import shard
from baremetalinferenceengine_b200.layer import WORKLOADS, LayerBuffers


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_weak_and_strong_partitions():
    for world in (1, 2, 3, 8):
        weak = [shard.weak_rows(r, world, 1000) for r in range(world)]
        assert [x.start for x in weak] == [1000 * r for r in range(world)]
        assert sum(len(x) for x in weak) == 1000 * world
        for total in (0, 1, 7, 131072, 131073):
            parts = [shard.strong_rows(r, world, total) for r in range(world)]
            covered = [i for p in parts for i in p]
            assert covered == list(range(total))
    with pytest.raises(ValueError):
        shard.weak_rows(2, 2, 10)


def test_max_over_ranks_without_group():
    assert shard.max_over_ranks([1.0, 3.0]) == [1.0, 3.0]


def _init(rank, world, port, timeout_s):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _shard_worker(rank, world, port, out_dir):
    _init(rank, world, port, 60)
    shape = WORKLOADS["tinyllama_fp32"].with_rows(512)
    rows = shard.weak_rows(rank, world, shape.rows)
    b = LayerBuffers(shape, "cpu", seed=7 + rank, row_offset=rows.start, with_table=False)
    # every rank's tokens are valid positions/sequences of its own cache
    assert int(b.positions.min()) >= 0 and int(b.positions.max()) < shape.max_seq
    assert int(b.seq_ids.min()) >= 0 and int(b.seq_ids.max()) < shape.num_seqs
    # global row ranges are disjoint and cover the job
    ranges = [None] * world
    dist.all_gather_object(ranges, (rows.start, rows.stop))
    covered = sorted(i for a, z in ranges for i in range(a, z))
    assert covered == list(range(world * shape.rows))
    # the timing reduction is a max over ranks
    got = shard.max_over_ranks([float(rank), 10.0 - rank])
    assert got == [float(world - 1), 10.0]
    dist.barrier()
    dist.destroy_process_group()
    open(os.path.join(out_dir, f"ok{rank}"), "w").close()


def test_two_gloo_ranks_partition_and_reduce(tmp_path):
    mp.start_processes(_shard_worker, args=(2, free_port(), str(tmp_path)), nprocs=2, start_method="spawn",
                       join=True)
    assert os.path.exists(tmp_path / "ok0") and os.path.exists(tmp_path / "ok1")


def _dying_worker(rank, world, port, out_dir):
    _init(rank, world, port, 5)
    if rank == 1:
        os._exit(3)  # leaves between steps, before the barrier, with nothing in flight
    try:
        dist.barrier()
        outcome = "barrier returned"
    except Exception as e:  # noqa: BLE001
        outcome = f"error: {type(e).__name__}"
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(outcome)
    os._exit(0)


def _strong_worker(rank, world, port, out_dir):
    """Fixed-total split: each rank builds only its block of the job's tokens;
    together the ranks write every (sequence, position) slot exactly once."""
    import dataclasses

    _init(rank, world, port, 60)
    job = dataclasses.replace(WORKLOADS["llama70b_bf16"], rows=1024, dim=32, hq=4, hkv=2, hd=8, ffn=16, vocab=64,
                              max_seq=256, num_seqs=4, dtype=torch.float32)
    local, rows = shard.local_shape(job, rank, world, "strong")
    b = LayerBuffers(local, "cpu", seed=7 + rank, row_offset=rows.start, with_table=False)
    assert b.q.shape[0] == len(rows) == local.rows
    assert int(b.seq_ids.max()) < local.num_seqs and int(b.positions.max()) < job.max_seq
    # back to global slots: the local sequence id is offset by the block's first sequence
    first_seq = rows.start // job.max_seq
    mine = [(first_seq + int(s), int(p)) for s, p in zip(b.seq_ids, b.positions)]
    every = [None] * world
    dist.all_gather_object(every, mine)
    slots = [x for part in every for x in part]
    assert len(slots) == len(set(slots)) == job.rows
    assert sorted(slots) == [(r // job.max_seq, r % job.max_seq) for r in range(job.rows)]
    # the parity flag is reduced the way bench.py reduces it: any failing rank fails the job
    flag = shard.max_over_ranks([1.0 if rank == world - 1 else 0.0])[0]
    assert flag == 1.0
    dist.barrier()
    dist.destroy_process_group()
    open(os.path.join(out_dir, f"ok{rank}"), "w").close()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_ranks_strong_split_cover_the_job_once(tmp_path, world):
    mp.start_processes(_strong_worker, args=(world, free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    assert all(os.path.exists(tmp_path / f"ok{r}") for r in range(world))


def test_a_dead_rank_is_detected_not_hung(tmp_path):
    ctx = mp.start_processes(_dying_worker, args=(2, free_port(), str(tmp_path)), nprocs=2, start_method="spawn",
                             join=False)
    for p in ctx.processes:
        p.join(timeout=120)
        assert not p.is_alive(), "a rank hung"
    assert ctx.processes[1].exitcode == 3
    assert (tmp_path / "rank0.txt").read_text().startswith("error"), "the survivor must see an error"


def test_layer_buffers_on_cpu_are_seeded_per_rank():
    shape = WORKLOADS["tinyllama_fp32"].with_rows(16)
    a = LayerBuffers(shape, "cpu", seed=1, with_table=False)
    b = LayerBuffers(shape, "cpu", seed=1, with_table=False)
    c = LayerBuffers(shape, "cpu", seed=2, with_table=False)
    assert torch.equal(a.q, b.q) and not torch.equal(a.q, c.q)

"""Host-side pieces of bench.py that run without a GPU: the CPU-baseline sample
sizing and timing (the oracle's layer step on all threads, and on one thread over
the first rows of the same sample, as the reference's loops run)."""
import bench
from baremetalinferenceengine_b200.layer import WORKLOADS


def test_sample_rows_stays_inside_the_workload_and_the_memory_cap():
    shape = WORKLOADS["llama70b_bf16"]
    per_row = 1e-3
    assert bench.sample_rows(shape, 16, 1.0, per_row) == 16000
    assert bench.sample_rows(shape, 16, 1e-9, per_row) == 16  # at least one token per thread
    assert bench.sample_rows(shape, 16, 1e9, per_row) <= shape.rows
    cap = int(bench.HOST_SAMPLE_BYTES // shape.with_rows(1).step_bytes())
    assert bench.sample_rows(shape, 16, 1e9, per_row) <= cap
    small = WORKLOADS["tinyllama_fp32"]
    assert bench.sample_rows(small, 64, 1e9, per_row) == small.rows


def test_cpu_baseline_reports_all_threads_and_one_thread_on_the_same_sample():
    shape = WORKLOADS["tinyllama_fp32"]
    gbs, rows, times, (gbs1, rows1, times1) = bench.cpu_baseline(shape, 2, 0.05, single_s=0.02)
    assert gbs > 0 and gbs1 > 0
    assert 1 <= rows1 <= rows <= shape.rows
    assert times and times1 and all(t > 0 for t in times + times1)
    # without the single-thread leg the result is the plain triple
    assert len(bench.cpu_baseline(shape, 2, 0.02)) == 3


def test_strong_split_shapes_and_config():
    """The default --scaling strong splits the job's 131072 70B tokens: 16384 per
    GPU at N=8, two whole sequences each; the config names the fixed total."""
    from baremetalinferenceengine_b200 import shard

    job = WORKLOADS["llama70b_bf16"]
    for world in (1, 2, 4, 8):
        parts = [shard.local_shape(job, r, world, "strong") for r in range(world)]
        assert sum(p.rows for p, _ in parts) == job.rows
        assert all(p.rows == job.rows // world and p.num_seqs == 16 // world for p, _ in parts)
        assert sum(p.step_bytes() for p, _ in parts) == job.step_bytes()
        c = bench.config_dict(job, world, "strong", parts[0][0])
        assert c["global_rows"] == 131072 and c["rows_per_gpu"] == 131072 // world
    weak = bench.config_dict(job, 8, "weak", job)
    assert weak["global_rows"] == 8 * 131072 and weak["rows_per_gpu"] == 131072
    # the 8B prefill job at N=8: half a sequence per GPU, one local cache sequence
    pre = WORKLOADS["llama8b_prefill_bf16"]
    p, rows = shard.local_shape(pre, 1, 8, "strong")
    assert (p.rows, p.num_seqs, rows.start) == (4096, 1, 4096)

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

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


def test_reference_kernel_step_binding():
    """The ctypes binding of the reference-kernel step (bench.py's GPU baseline
    leg) matches the C function: a call over zero tokens issues nothing and needs
    no GPU."""
    import os

    from oracle import oracle as orc

    if not os.path.exists(orc.REF_KERNELS_LIB):
        import pytest

        pytest.skip("oracle/_ref/libref_kernels.so is not built")
    L = bench.ref_kernels_lib()
    args = [31, 0, None, None, None] + [None] * 16 + [4096, 32, 8, 128, 14336, 8192] + [5e5, 1e-5]
    assert L.ref_layer_step_rows(*args) == 0


def test_run_step_uses_one_launch_for_decode_batches():
    """Layer steps of at most 512 tokens go through bm_layer_step's single launch;
    their kernel list is that one launch, their metric still the five ops' bytes."""
    from baremetalinferenceengine_b200 import layer

    dec = WORKLOADS["llama8b_decode_bf16"]
    assert dec.fused and WORKLOADS["tinyllama_fp32"].fused
    assert not WORKLOADS["llama70b_bf16"].fused and not WORKLOADS["swiglu_stress_bf16"].fused
    assert [k for k, _ in dec.step_kernels()] == ["layer_step"]
    b = dec.bytes_per_row()
    assert dec.step_bytes() == (b["embed_gather"] + 2 * b["add_rmsnorm"] + b["rope_kv_store"] + b["swiglu"]) * 64
    assert dec.step_kernels()[0][1] < dec.step_bytes()  # the single launch moves fewer bytes
    assert layer.FUSED_MAX_ROWS == 512
    big = WORKLOADS["llama70b_bf16"]
    assert sum(n for _, n in big.step_kernels()) == big.step_bytes()


def test_packed_step_buffers_are_two_contiguous_ranges():
    """A decode-sized step keeps its tensors in one arena: the inputs (q last) form
    [0, in_end), the outputs (q first) [out_start, end), each tensor at a 256-byte
    boundary, with the same seeded values as separate buffers; with_arena binds the
    same step to a second arena and shares everything else."""
    import torch

    from baremetalinferenceengine_b200 import layer

    for name in ("llama8b_decode_bf16", "tinyllama_fp32", "swiglu_stress_bf16"):
        shape = WORKLOADS[name].with_rows(24)
        b = layer.LayerBuffers(shape, "cpu", seed=5, with_table=False, packed=True)
        plain = layer.LayerBuffers(shape, "cpu", seed=5, with_table=False)
        base = b.arena.data_ptr()
        spans = {}
        for n in set(b.inputs()) | set(b.outputs()):
            t = getattr(b, n)
            off = t.data_ptr() - base
            assert off % 256 == 0 and t.is_contiguous()
            spans[n] = (off, off + t.numel() * t.element_size())
        for n in b.inputs():
            assert spans[n][1] <= b.in_end
            assert torch.equal(getattr(b, n), getattr(plain, n))
        for n in b.outputs():
            assert spans[n][0] >= b.out_start and spans[n][1] <= b.arena.numel()
        assert b.out_start <= b.in_end  # q (when the step has it) lies in both ranges
        other = b.with_arena(torch.zeros_like(b.arena))
        assert other.embed is b.embed and other.k_cache is b.k_cache and other.status is b.status
        assert all(getattr(other, n).data_ptr() != getattr(b, n).data_ptr() for n in spans)

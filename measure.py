"""Throughput of the tensor-core rows: decode attention and the fused FFN GEMM.

    python measure.py attention [--shapes a,b] [--reps 50] [--once]
    python measure.py ffn       [--shapes a,b] [--reps 20] [--once]

One JSON line per shape on stdout. Inputs are seeded synthetic tensors of the
Llama-3 8B / 70B decode and prefill shapes, resident on the GPU. The call is
captured once in a CUDA graph (so the timed window holds GPU work only, not the
host's launch path); each replay is preceded by a 256 MB write that evicts L2
and timed alone with CUDA events on its stream (the mean of the middle 80 % of --reps:
the B200's event timestamps advance in 2.05 µs steps, so a median of a ~20 µs call is
one of a few values, while the mean of many replays, each starting at a different
phase of the timer, resolves far below a step). That write
leaves L2 full of dirty lines, which the timed call then writes back as it
misses (up to 126 MB: ~19 us of DRAM time, a large share of a short call), so
every shape is also timed after the write followed by a 256 MB read of another
buffer, which leaves L2 holding clean lines only (``ms_clean_l2``). ``--once``
makes two untimed calls per shape and nothing else (for profilers).

attention: algorithmic bytes = the K and V rows every query reads plus q and the
    output; roofline = HBM (hbm_gbs of MEASURED_PEAKS.json, else 6650 GB/s).
ffn: bm_gemm_swiglu, FLOPs = 2 * rows * dim * hidden * 2; roofline = tensor
    (bf16_tflops of MEASURED_PEAKS.json, the burst figure, else 1590 TFLOP/s),
    with torch.matmul (cuBLAS) + silu * up on the same tensors timed beside it.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import torch  # noqa: E402

from baremetalinferenceengine_b200 import _lib, ops  # noqa: E402
FLUSH_BYTES = 256 << 20

# name: (batch, q heads, kv heads, head_dim, max_seq, lengths "full" or "uniform", dtype)
ATTENTION_SHAPES = {
    "8b_decode_b64_full": (64, 32, 8, 128, 8192, "full", torch.bfloat16),
    "8b_decode_b64_ragged": (64, 32, 8, 128, 8192, "uniform", torch.bfloat16),
    "70b_decode_b64_full": (64, 64, 8, 128, 8192, "full", torch.bfloat16),
    "70b_decode_b16_ragged": (16, 64, 8, 128, 8192, "uniform", torch.bfloat16),
    "8b_single_sequence": (1, 32, 8, 128, 8192, "full", torch.bfloat16),
    "8b_decode_b2_full": (2, 32, 8, 128, 8192, "full", torch.bfloat16),
    "70b_decode_b2_ragged": (2, 64, 8, 128, 8192, "uniform", torch.bfloat16),
    "8b_decode_b64_full_fp32": (64, 32, 8, 128, 8192, "full", torch.float32),
}
# name: (rows, dim, hidden)
FFN_SHAPES = {
    "8b_prefill_32768": (32768, 4096, 14336),
    "8b_prefill_8192": (8192, 4096, 14336),
    "8b_decode_64": (64, 4096, 14336),
    "70b_prefill_16384": (16384, 8192, 28672),
    "70b_prefill_4096": (4096, 8192, 28672),
}


def peaks():
    """(hbm GB/s, source), (bf16 TFLOP/s, source) from MEASURED_PEAKS.json or the fallbacks."""
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return (float(p["hbm_gbs"]), "measured"), (float(p["bf16_tflops"]), "measured burst")
    except (OSError, KeyError, ValueError):
        return (6650.0, "fallback"), (1590.0, "fallback")


def trimmed_mean(times, cut: float = 0.1) -> float:
    """Mean of the values left after dropping the lowest and highest `cut` share."""
    t = sorted(times)
    k = int(len(t) * cut)
    t = t[k:len(t) - k] or t
    return sum(t) / len(t)


def time_call(fn, reps: int, dev, clean: bool = False) -> float:
    """Milliseconds of one replay of fn() captured as a CUDA graph (trimmed mean
    over reps replays), each after an L2-evicting write (clean: the write, then a
    read of another buffer larger than L2, so no dirty line is left to write back)."""
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    reread = torch.ones(FLUSH_BYTES // 4, dtype=torch.float32, device=dev) if clean else None
    for _ in range(3):
        fn()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch.cuda.Stream(dev)):
        fn()
    graph.replay()
    torch.cuda.synchronize(dev)
    times = []
    for _ in range(reps):
        flush.zero_()
        if clean:
            reread.sum()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    return trimmed_mean(times)


def attention(names, reps: int, once: bool, dev) -> None:
    L = _lib.load()
    (hbm, hbm_src), _ = peaks()
    for name in names:
        batch, hq, hkv, hd, max_seq, kind, dt = ATTENTION_SHAPES[name]
        g = torch.Generator(device=dev)
        g.manual_seed(0)
        kc = torch.randn(batch, hkv, max_seq, hd, device=dev, generator=g).to(dt)
        vc = torch.randn(batch, hkv, max_seq, hd, device=dev, generator=g).to(dt)
        q = torch.randn(batch, hq, hd, device=dev, generator=g).to(dt)
        out = torch.empty_like(q)
        if kind == "full":
            lens = torch.full((batch,), max_seq, dtype=torch.int32, device=dev)
        else:
            lens = torch.randint(1, max_seq + 1, (batch,), generator=g, device=dev, dtype=torch.int32)
        seq_ids = torch.arange(batch, dtype=torch.int32, device=dev)
        need = ctypes.c_size_t()
        _lib.check(L.bm_decode_attention_workspace_size(batch, hq, hkv, hd, max_seq, ctypes.byref(need)))
        ws = torch.empty(max(1, need.value), dtype=torch.uint8, device=dev)
        status = ops.DeviceStatus(dev)

        def call():
            _lib.check(L.bm_decode_attention(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                             seq_ids.data_ptr(), lens.data_ptr(), max_seq, batch, hq, hkv, hd,
                                             max_seq, batch, 0.0, ws.data_ptr(), need.value, ops.bm_dtype(q),
                                             status.ptr, torch.cuda.current_stream(dev).cuda_stream))

        if once:
            call()
            call()
            torch.cuda.synchronize(dev)
            assert status.read() == 0
            continue
        ms = time_call(call, reps, dev)
        ms_clean = time_call(call, reps, dev, clean=True)
        assert status.read() == 0, "device status set"
        es = q.element_size()
        nbytes = int(lens.sum().item()) * hkv * hd * es * 2 + 2 * q.numel() * es
        gbs = nbytes / (ms / 1e3) / 1e9
        print(json.dumps({
            "row": "decode_attention", "shape": name, "batch": batch, "q_heads": hq, "kv_heads": hkv,
            "head_dim": hd, "max_seq": max_seq, "lengths": kind, "dtype": "bf16" if es == 2 else "f32",
            "kernel": "tcgen05" if es == 2 and hd == 128 else "cuda cores",
            "ms": round(ms, 4), "algorithmic_bytes": nbytes, "gbs": round(gbs, 1),
            "roofline": {"bound": "hbm", "peak": hbm, "peak_source": hbm_src, "frac": round(gbs / hbm, 4)},
            "ms_clean_l2": round(ms_clean, 4), "frac_clean_l2": round(nbytes / (ms_clean / 1e3) / 1e9 / hbm, 4),
            "l2": "flushed before each call (a 256 MB write; ms_clean_l2: the write and a 256 MB read)",
            "timing": "CUDA-graph replay"}), flush=True)
        del kc, vc
        torch.cuda.empty_cache()


def ffn(names, reps: int, once: bool, dev) -> None:
    _, (tf_peak, tf_src) = peaks()
    for name in names:
        rows, dim, hidden = FFN_SHAPES[name]
        g = torch.Generator(device=dev)
        g.manual_seed(0)
        x = torch.randn(rows, dim, device=dev, generator=g).to(torch.bfloat16)
        wg = (torch.randn(dim, hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        wu = (torch.randn(dim, hidden, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        out = torch.empty(rows, hidden, device=dev, dtype=torch.bfloat16)
        status = ops.DeviceStatus(dev)

        def call():
            ops.gemm_swiglu(x, wg, wu, out=out, status=status)

        if once:
            call()
            call()
            torch.cuda.synchronize(dev)
            assert status.read() == 0
            continue
        ms = time_call(call, reps, dev)
        ms_clean = time_call(call, reps, dev, clean=True)
        assert status.read() == 0, "device status set"
        cublas = lambda: torch.nn.functional.silu(x @ wg) * (x @ wu)  # noqa: E731
        cublas_ms = time_call(cublas, reps, dev)
        cublas_ms_clean = time_call(cublas, reps, dev, clean=True)
        flops = 2.0 * rows * dim * hidden * 2
        nbytes = (rows * dim + 2 * dim * hidden + rows * hidden) * 2
        tflops = flops / (ms / 1e3) / 1e12
        print(json.dumps({
            "row": "ffn_gemm_swiglu", "shape": name, "rows": rows, "dim": dim, "hidden": hidden, "dtype": "bf16",
            "ms": round(ms, 4), "tflops": round(tflops, 1), "algorithmic_bytes": nbytes,
            "gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
            "roofline": {"bound": "tensor", "peak": tf_peak, "peak_source": tf_src,
                         "frac": round(tflops / tf_peak, 4)},
            "cublas_matmul_plus_swiglu_ms": round(cublas_ms, 4),
            "cublas_tflops": round(flops / (cublas_ms / 1e3) / 1e12, 1),
            "ms_clean_l2": round(ms_clean, 4), "gbs_clean_l2": round(nbytes / (ms_clean / 1e3) / 1e9, 1),
            "cublas_ms_clean_l2": round(cublas_ms_clean, 4),
            "l2": "flushed before each call (a 256 MB write; *_clean_l2: the write and a 256 MB read)",
            "timing": "CUDA-graph replay"}), flush=True)
        del x, wg, wu, out
        torch.cuda.empty_cache()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("row", choices=["attention", "ffn"])
    ap.add_argument("--shapes", default="", help="comma-separated subset (default: all)")
    ap.add_argument("--reps", type=int, default=0)
    ap.add_argument("--once", action="store_true")
    args = ap.parse_args(argv)
    assert torch.cuda.is_available(), "measure needs a CUDA device"
    dev = torch.device("cuda", 0)
    table = ATTENTION_SHAPES if args.row == "attention" else FFN_SHAPES
    names = [s for s in args.shapes.split(",") if s] or list(table)
    for n in names:
        if n not in table:
            raise SystemExit(f"unknown shape {n}; choose from {', '.join(table)}")
    if args.row == "attention":
        attention(names, args.reps or 50, args.once, dev)
    else:
        ffn(names, args.reps or 20, args.once, dev)
    return 0


if __name__ == "__main__":
    sys.exit(main())

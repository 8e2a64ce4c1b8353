#!/usr/bin/env python
"""Throughput of the fused layer-op kernels on B200: one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload llama70b_bf16] [--rows R] [--e2e-steps E]

A step is one layer's memory-bound ops over one batch of tokens, issued through
the C ABI: embedding gather -> residual add + RMSNorm -> RoPE on Q/K with the
K/V write into the static cache -> residual add + RMSNorm -> SwiGLU
(baremetalinferenceengine_b200.layer). The default workload is the
Llama-3-70B shape: 131072 tokens (16 sequences x 8192 positions), dim 8192,
64 Q / 8 KV heads of 128, FFN 28672, bf16 — 49 GB of algorithmic traffic per
step, far above the 126 MB L2, so no flush is needed between steps.

N > 1 runs one process per GPU (torchrun); the workload's tokens are one job
split into contiguous blocks of ceil(R/N), one per rank (strong scaling, the
default; --scaling weak gives every rank its own copy of the batch). Rows are
independent: no collectives on the data path. Time is the max over ranks of the
CUDA-event time of exactly K steps, bracketed by a barrier and a synchronize.

value: whole-job algorithmic HBM GB/s (bytes every kernel must move / time).
e2e:   the same metric with the step's inputs copied in from pinned host memory
       and its outputs copied back, every step, inside the timed region.
--impl reference: the CPU implementation (the oracle: the reference's
       double-precision check loops restated in C, pinned bit-for-bit to them)
       on all host cores, over a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "achieved HBM GB/s and % of B200 peak per fused layer kernel; rows/s at 1/2/4/8 GPUs"
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 2**20
L2_RESIDENT_BYTES = 4 * L2_BYTES  # a step moving less than this would be served from L2 when repeated
L2_FLUSH_BYTES = 256 * 2**20


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def parse_args():
    from baremetalinferenceengine_b200.layer import WORKLOADS

    ap = argparse.ArgumentParser(description="fused layer-op kernel benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(OP_ROWS), default="llama70b_bf16",
                    help="a layer-step workload (default) or one of the tensor-core op rows")
    ap.add_argument("--rows", type=int, default=0, help="override the workload's tokens")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="strong: the workload's tokens split across the GPUs (default); weak: every GPU its own copy")
    ap.add_argument("--no-parity", action="store_true", help="skip the sampled-row oracle check after timing")
    ap.add_argument("--no-ref-gpu", action="store_true", help="skip timing the reference's CUDA kernels")
    ap.add_argument("--ref-gpu-rows", type=int, default=256, help="tokens of the reference-kernel sample")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--e2e-chunks", type=int, default=16)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="target CPU-baseline sample time")
    return ap.parse_args()


def measured_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            peaks = json.load(f)
        return float(peaks["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ----------------------------------------------------------------------------- clocks

NVML_REASONS = {
    0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting", 0x10: "sync_boost",
}


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML (read-only) while running."""

    def __init__(self, torch_device, period_s: float = 0.002):
        self.samples, self.period, self.err = [], period_s, None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            import torch

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(torch_device).uuid)
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 - report, do not fail the benchmark
            self.err = f"{type(e).__name__}: {e}"

    def _run(self):
        p, h = self.nvml, self.handle
        while not self._stop.is_set():
            try:
                sm = p.nvmlDeviceGetClockInfo(h, p.NVML_CLOCK_SM)
                get = getattr(p, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    p.nvmlDeviceGetCurrentClocksThrottleReasons
                reasons = get(h)
                self.samples.append((sm, reasons))
            except Exception as e:  # noqa: BLE001
                self.err = str(e)
                return
            time.sleep(self.period)

    def __enter__(self):
        if self.err is None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        if self.err is not None and not self.samples:
            return {"unavailable": self.err}
        mask = 0
        for _, r in self.samples:
            mask |= r
        reasons = sorted(name for bit, name in NVML_REASONS.items() if mask & bit)
        return {"sm_mhz": statistics.median(s for s, _ in self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples),
                "source": f"NVML every {self.period * 1e3:g} ms during the timed region"}


# ----------------------------------------------------------------------------- CPU side (oracle)

def make_host_step(shape, rows: int, seed: int = 0):
    """Host buffers of `rows` tokens of `shape` for the CPU implementation (the
    oracle's layer step). Values are tiled from a seeded N(0,1) block."""
    import numpy as np

    from oracle import oracle as orc

    rng = np.random.default_rng(seed)
    block = rng.standard_normal(1 << 22).astype(np.float32)
    is_bf16 = shape.es == 2
    if is_bf16:
        block = orc.f32_to_bf16(block)
    dt = np.uint16 if is_bf16 else np.float32

    def fill(n, scale=1.0, offset=0.0):
        src = block
        if scale != 1.0 or offset != 0.0:
            f = (orc.bf16_to_f32(block) if is_bf16 else block) * scale + offset
            src = orc.f32_to_bf16(f) if is_bf16 else f.astype(np.float32)
        out = np.empty(n, dt)
        for i in range(0, n, src.size):
            m = min(src.size, n - i)
            out[i:i + m] = src[:m]
        return out

    R, D = rows, shape.dim
    bufs = {
        "ids": rng.integers(0, shape.vocab, R, dtype=np.int32),
        "embed": fill(shape.vocab * D, 0.02),
        "hidden": np.empty(R * D, dt),
        "attn_out": fill(R * D),
        "w_attn": fill(D, 0.02, 1.0),
        "normed": np.empty(R * D, dt),
        "q": fill(R * shape.hq * shape.hd),
        "k": fill(R * shape.hkv * shape.hd),
        "v": fill(R * shape.hkv * shape.hd),
        "k_cache": np.zeros(shape.num_seqs * shape.hkv * shape.max_seq * shape.hd, dt),
        "v_cache": np.zeros(shape.num_seqs * shape.hkv * shape.max_seq * shape.hd, dt),
        "ffn_out": fill(R * D),
        "w_ffn": fill(D, 0.02, 1.0),
        "gate": fill(R * shape.ffn),
        "up": fill(R * shape.ffn),
        "act": np.empty(R * shape.ffn, dt),
    }
    if shape.positions == "uniform":
        bufs["positions"] = rng.integers(0, shape.max_seq, R, dtype=np.int32)
        bufs["seq_ids"] = (np.arange(R) % shape.num_seqs).astype(np.int32)
    else:
        r = np.arange(R, dtype=np.int64)
        bufs["positions"] = (r % shape.max_seq).astype(np.int32)
        bufs["seq_ids"] = ((r // shape.max_seq) % shape.num_seqs).astype(np.int32)
    st = orc.OracleStep()
    st.rows, st.dim, st.vocab, st.ffn = R, D, shape.vocab, shape.ffn
    st.hq, st.hkv, st.hd, st.max_seq, st.num_seqs, st.table_len = (shape.hq, shape.hkv, shape.hd, shape.max_seq,
                                                                   shape.num_seqs, 0)
    st.eps, st.theta, st.dtype = shape.eps, shape.theta, 1 if is_bf16 else 0
    st.ops = 1 | 16 if shape.kind == "stress" else 0  # stress: gather + SwiGLU; else all five ops
    for name, arr in bufs.items():
        setattr(st, name, arr.ctypes.data)
    return st, bufs


def seconds_per_row(shape) -> float:
    """One thread's time for one token of the CPU layer step (8-token probe; a small
    vocabulary keeps the probe's embedding table small, the per-token work is the same)."""
    import dataclasses

    from oracle import oracle as orc

    probe = dataclasses.replace(shape, vocab=min(shape.vocab, 1024))
    calib = min(shape.rows, 8)
    st, keep = make_host_step(probe, calib)
    orc.layer_step(st, 0, calib, 1)
    t0 = time.perf_counter()
    orc.layer_step(st, 0, calib, 1)
    del keep
    return max((time.perf_counter() - t0) / calib, 1e-7)


HOST_SAMPLE_BYTES = 8e9  # cap on the CPU sample's host buffers


def sample_rows(shape, threads: int, seconds: float, per_row: float) -> int:
    """Tokens the CPU sample covers: about `seconds` of work on `threads` threads,
    at least one per thread, within the workload and the host-memory cap."""
    by_mem = int(HOST_SAMPLE_BYTES // max(1, shape.with_rows(1).step_bytes()))
    return int(max(1, min(shape.rows, by_mem, max(threads, seconds * threads / per_row))))


def cpu_baseline(shape, threads: int, target_s: float, single_s: float = 0.0):
    """Times the oracle's layer step on a bounded row sample with `threads` host
    threads, repeating the sample until about `target_s` of work is timed.
    Returns (GB/s, rows sampled, seconds per repetition). With single_s > 0 it also
    times one thread on the first rows of the same sample (about single_s of work)
    and returns that triple as a fourth item."""
    from oracle import oracle as orc

    per_row = seconds_per_row(shape)
    rows = sample_rows(shape, threads, target_s, per_row)
    st, keep = make_host_step(shape, rows)

    def timed(n, nthreads, budget):
        orc.layer_step(st, 0, n, nthreads)  # warm the pages
        times = []
        while not times or (sum(times) < budget and len(times) < 50):
            t0 = time.perf_counter()
            bad = orc.layer_step(st, 0, n, nthreads)
            times.append(time.perf_counter() - t0)
            assert bad == 0, bad
        return shape.with_rows(n).step_bytes() / statistics.median(times) / 1e9, n, times

    result = timed(rows, threads, target_s)
    if single_s > 0:
        return result + (timed(min(rows, sample_rows(shape, 1, single_s, per_row)), 1, single_s),)
    return result


def run_reference(args, shape):
    """--impl reference: rank 0 times the CPU implementation; other ranks exit."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = host_threads()
    K, W = args.steps, args.warmup
    # each step is a bounded sample sized so the whole run takes about two minutes
    per_step = max(0.5, 90.0 / max(1, K + W))
    from oracle import oracle as orc

    rows = sample_rows(shape, threads, per_step, seconds_per_row(shape))
    st, keep = make_host_step(shape, rows)
    for _ in range(W):
        orc.layer_step(st, 0, rows, threads)
    t0 = time.perf_counter()
    for _ in range(K):
        orc.layer_step(st, 0, rows, threads)
    elapsed = time.perf_counter() - t0
    sample_bytes = shape.with_rows(rows).step_bytes()
    value = sample_bytes * K / elapsed / 1e9
    sample = (f"{rows} of {shape.rows} tokens of one {shape.name} layer step per step (gather, add+RMSNorm, "
              f"RoPE+KV store, add+RMSNorm, SwiGLU), oracle_layer_step_mt on {threads} threads")
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": K, "warmup": W,
        "ms_per_step": round(elapsed / K * 1e3, 3), "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "bf16" if shape.es == 2 else "f32", "data": "synthetic (seeded N(0,1))",
        "impl": "reference",
        "config": config_dict(shape, args.gpus, args.scaling, shard_of(shape, args)),
        "rows_per_s": round(rows * K / elapsed, 1),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def shard_of(shape, args):
    """Rank 0's share of the workload (its config entry), without a process group."""
    from baremetalinferenceengine_b200 import shard

    return shard.local_shape(shape, 0, max(1, args.gpus), args.scaling)[0]


def config_dict(shape, n, scaling="weak", local=None):
    """The workload `shape` (the whole job's tokens for strong scaling, each GPU's
    for weak) and this rank's share `local`."""
    local = local or shape
    strong = scaling == "strong"
    return {"workload": shape.name, "description": shape.description, "rows_per_gpu": local.rows,
            "global_rows": shape.rows if strong else shape.rows * n, "dim": shape.dim, "q_heads": shape.hq,
            "kv_heads": shape.hkv, "head_dim": shape.hd, "ffn": shape.ffn, "vocab": shape.vocab,
            "rope_theta": shape.theta, "max_seq": shape.max_seq, "sequences": shape.num_seqs * (1 if strong else n),
            "sequences_per_gpu": local.num_seqs,
            "l2": f"inputs larger than L2: {local.step_bytes() / 1e9:.2f} GB moved per step per GPU vs 126 MB L2; "
                  "the step is one CUDA graph replayed back to back; per-kernel times from steps launched one "
                  "kernel at a time with events between launches"
                  if local.step_bytes() >= L2_RESIDENT_BYTES else
                  "L2-resident working set: the step is one CUDA graph replayed after a 256 MB write that "
                  "flushes L2; per-kernel times are per launch of a 16-launch graph (L2 warm)",
            "parallelism": (f"rows{n}: the job's {shape.rows} tokens split into {n} contiguous block(s) of "
                            f"ceil({shape.rows}/{n}) = {-(-shape.rows // n)}, one per GPU, no collectives")
            if strong else f"rows{n}: every GPU its own {shape.rows} tokens (weak scaling), no collectives"}


# ----------------------------------------------------------------------------- op rows
# The two contractions beyond the layer-op path, each as its own bench line with
# the same contract: decode attention over a resident KV cache, and the FFN
# front half (two projections + SwiGLU). A step is one call over one batch.

OP_ROWS = {
    "attention_8b_decode_b64_bf16": dict(kind="attention", batch=64, hq=32, hkv=8, hd=128, max_seq=8192,
                                         dtype="bf16", description="Llama-3-8B decode attention: 64 queries, "
                                         "32 Q / 8 KV heads of 128, 8192 cached positions each"),
    "attention_8b_decode_b64_f32": dict(kind="attention", batch=64, hq=32, hkv=8, hd=128, max_seq=8192,
                                        dtype="f32", description="the same in fp32"),
    "attention_70b_decode_b64_bf16": dict(kind="attention", batch=64, hq=64, hkv=8, hd=128, max_seq=8192,
                                          dtype="bf16", description="Llama-3-70B decode attention: 64 queries, "
                                          "64 Q / 8 KV heads of 128, 8192 cached positions each"),
    "ffn_gemm_swiglu_8b_prefill_bf16": dict(kind="ffn", rows=32768, dim=4096, hidden=14336, dtype="bf16",
                                            description="Llama-3-8B FFN front half over 32768 prefill tokens: "
                                            "silu(x Wg) * (x Wu), dim 4096, hidden 14336"),
    "ffn_gemm_swiglu_70b_prefill_bf16": dict(kind="ffn", rows=16384, dim=8192, hidden=28672, dtype="bf16",
                                             description="Llama-3-70B FFN front half over 16384 prefill tokens"),
}
OP_METRIC = {"attention": ("decode attention: algorithmic HBM GB/s of K/V read", "GB/s"),
             "ffn": ("fused GEMM + SwiGLU: TFLOP/s", "TFLOP/s")}


def measured_bf16_peak():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, 1400.0, "fallback"


class OpRow:
    """Device inputs of one op row and its call through the public API."""

    def __init__(self, spec, dev, seed):
        import ctypes

        import torch

        from baremetalinferenceengine_b200 import _lib, ops
        self.spec, self.dev = spec, dev
        self.dt = torch.bfloat16 if spec["dtype"] == "bf16" else torch.float32
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        self.status = ops.DeviceStatus(dev)
        if spec["kind"] == "attention":
            b, hq, hkv, hd, S = spec["batch"], spec["hq"], spec["hkv"], spec["hd"], spec["max_seq"]
            self.kc = torch.randn(b, hkv, S, hd, device=dev, generator=g).to(self.dt)
            self.vc = torch.randn(b, hkv, S, hd, device=dev, generator=g).to(self.dt)
            self.q = torch.randn(b, hq, hd, device=dev, generator=g).to(self.dt)
            self.out = torch.empty_like(self.q)
            self.lens = torch.full((b,), S, dtype=torch.int32, device=dev)
            self.seq = torch.arange(b, dtype=torch.int32, device=dev)
            L = _lib.load()
            need = ctypes.c_size_t()
            _lib.check(L.bm_decode_attention_workspace_size(b, hq, hkv, hd, S, ctypes.byref(need)))
            self.need = need.value
            self.ws = torch.empty(max(1, need.value), dtype=torch.uint8, device=dev)
            es = self.q.element_size()
            self.bytes = b * S * hkv * hd * es * 2 + 2 * self.q.numel() * es
            self.units = self.bytes / 1e9  # GB per step
            self.launches = 1 + (1 if need.value > 0 else 0)
            self.inputs, self.outputs = [self.q], [self.out]
        else:
            r, d, h = spec["rows"], spec["dim"], spec["hidden"]
            self.x = torch.randn(r, d, device=dev, generator=g).to(self.dt)
            self.wg = (torch.randn(d, h, device=dev, generator=g) * 0.02).to(self.dt)
            self.wu = (torch.randn(d, h, device=dev, generator=g) * 0.02).to(self.dt)
            self.out = torch.empty(r, h, device=dev, dtype=self.dt)
            self.flops = 4.0 * r * d * h
            self.units = self.flops / 1e12  # TFLOP per step
            self.launches = 1
            self.inputs, self.outputs = [self.x], [self.out]

    def call(self, stream):
        import torch

        from baremetalinferenceengine_b200 import _lib, ops
        sp = self.spec
        if sp["kind"] == "attention":
            L = _lib.load()
            _lib.check(L.bm_decode_attention(
                self.out.data_ptr(), self.q.data_ptr(), self.kc.data_ptr(), self.vc.data_ptr(), self.seq.data_ptr(),
                self.lens.data_ptr(), sp["max_seq"], sp["batch"], sp["hq"], sp["hkv"], sp["hd"], sp["max_seq"],
                sp["batch"], 0.0, self.ws.data_ptr(), self.need, ops.bm_dtype(self.q), self.status.ptr,
                stream.cuda_stream))
        else:
            with torch.cuda.stream(stream):
                ops.gemm_swiglu(self.x, self.wg, self.wu, out=self.out, status=self.status, stream=stream)


def cpu_op_row(spec, threads: int, target_s: float, reps: int = 0, warmup: int = 0):
    """The oracle on a bounded sample: one call per host thread (a query's
    attention, or one row of the FFN), repeated to about target_s (or exactly
    `reps` times after `warmup`). Returns (value in the row's unit, sample
    description, wall seconds per repetition)."""
    import numpy as np

    from oracle import oracle as orc
    rng = np.random.default_rng(7)
    bf16 = spec["dtype"] == "bf16"

    def host(shape, scale=1.0):
        x = (rng.standard_normal(shape, dtype=np.float32) * scale)
        return orc.f32_to_bf16(x) if bf16 else x

    if spec["kind"] == "attention":
        hq, hkv, hd, S = spec["hq"], spec["hkv"], spec["hd"], spec["max_seq"]
        per = [(host((1, hq, hd)), host((1, hkv, S, hd)), host((1, hkv, S, hd)), np.zeros((1, hq, hd),
                np.uint16 if bf16 else np.float32)) for _ in range(threads)]
        lens = np.full(1, S, np.int32)
        L = orc.lib()

        def job(i):
            q, k, v, o = per[i]
            return lambda: L.oracle_decode_attention(o.ctypes.data, q.ctypes.data, k.ctypes.data, v.ctypes.data,
                                                     None, lens.ctypes.data, 1, hq, hkv, hd, S, 1, 0 if not bf16 else 1)
        jobs = [job(i) for i in range(threads)]
        unit_per_rep = threads * (S * hkv * hd * (2 if bf16 else 4) * 2) / 1e9
        sample = f"{threads} of {spec['batch']} queries (full 8192-position caches), oracle_decode_attention, one per thread"
    else:
        d, h = spec["dim"], spec["hidden"]
        wg, wu = host((d, h), 0.02), host((d, h), 0.02)
        xs = [host((1, d)) for _ in range(threads)]
        outs = [np.zeros((1, h), wg.dtype) for _ in range(threads)]
        L = orc.lib()

        def job(i):
            return lambda: L.oracle_gemm_swiglu(outs[i].ctypes.data, xs[i].ctypes.data, wg.ctypes.data,
                                                wu.ctypes.data, 1, d, h, 1 if bf16 else 0, 1)
        jobs = [job(i) for i in range(threads)]
        unit_per_rep = threads * 4.0 * d * h / 1e12
        sample = f"{threads} of {spec['rows']} rows, oracle_gemm_swiglu, one row per thread"
    def once():
        ths = [threading.Thread(target=j) for j in jobs]
        t0 = time.perf_counter()
        for t in ths:
            t.start()
        for t in ths:
            t.join()
        return time.perf_counter() - t0

    for _ in range(warmup):
        once()
    times = []
    while (len(times) < reps) if reps else (not times or (sum(times) < target_s and len(times) < 20)):
        times.append(once())
    return unit_per_rep / statistics.median(times), sample, times


def op_row_config(name, spec, n):
    c = {"workload": name, "description": spec["description"], "parallelism":
         f"rows{n}: each GPU its own instance (weak scaling), no collectives",
         "l2": "inputs larger than L2 (> 1 GB per step): no flush needed"}
    c.update({k: v for k, v in spec.items() if k not in ("description",)})
    return c


def run_op_row(args) -> int:
    spec = OP_ROWS[args.workload]
    metric, unit = OP_METRIC[spec["kind"]]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    K, W = args.steps, args.warmup
    if args.impl == "reference":
        if rank != 0:
            return 0
        threads = host_threads()
        value, sample, times = cpu_op_row(spec, threads, 0.0, reps=K, warmup=W)
        value = sum(times) and (value * statistics.median(times) * len(times) / sum(times))  # K steps / total time
        line = {"metric": metric, "value": round(value, 4), "unit": unit, "n_gpus": args.gpus, "steps": K,
                "warmup": W, "ms_per_step": round(sum(times) / K * 1e3, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": spec["dtype"], "data": "synthetic (seeded N(0,1))",
                "impl": "reference", "config": op_row_config(args.workload, spec, args.gpus),
                "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": threads, "kind": "port",
                                 "sample": sample},
                "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    import torch.distributed as dist

    from baremetalinferenceengine_b200 import shard
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        log(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 under torchrun")
        return 2
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    row = OpRow(spec, dev, seed=2000 + rank)
    stream = torch.cuda.Stream(dev)
    for _ in range(W):
        row.call(stream)
    stream.synchronize()
    assert row.status.read(stream) == 0, "device status set during warm-up"
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(dev) as clocks:
        for i in range(K):
            ev[i][0].record(stream)
            row.call(stream)
            ev[i][1].record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    assert row.status.read(stream) == 0, "device status set during the timed steps"
    per_step = [e0.elapsed_time(e1) for e0, e1 in ev]
    elapsed_ms = shard.max_over_ranks([sum(per_step)], device=dev)[0]
    value = world * row.units * K / (elapsed_ms / 1e3)
    mean_ms = elapsed_ms / K
    if spec["kind"] == "attention":
        peak, kind = measured_peak()
        achieved = row.bytes / (mean_ms / 1e3) / 1e9
        roofline = {"kernel": "bm_decode_attention", "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                    "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                    "peak_source": f"{kind} hbm_gbs", "algorithmic_bytes_per_launch": row.bytes}
    else:
        burst, sustained, kind = measured_bf16_peak()
        achieved = row.flops / (mean_ms / 1e3) / 1e12
        roofline = {"kernel": "bm_gemm_swiglu", "bound": "tensor", "achieved": round(achieved, 1), "peak": burst,
                    "unit": "TFLOP/s", "frac": round(achieved / burst, 4), "frac_of_sustained":
                    round(achieved / sustained, 4), "traffic": None, "peak_source": f"{kind} bf16_tflops (burst)",
                    "algorithmic_flops_per_launch": row.flops}
    line = {"metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(mean_ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": spec["dtype"], "data": "synthetic: seeded N(0,1) caches / activations, N(0,0.02) weights",
            "impl": "ours", "config": op_row_config(args.workload, spec, world), "roofline": roofline,
            "gpu_launches": row.launches * K, "clocks": clocks.summary() if rank == 0 else None}
    if not args.no_e2e:
        # the resident state (cache or weights) stays on the device; each step's
        # inputs come from pinned host memory and its output goes back
        h_in = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in row.inputs]
        h_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in row.outputs]
        for h, t in zip(h_in, row.inputs):
            h.copy_(t)
        E = max(1, args.e2e_steps)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(E):
                for h, t in zip(h_in, row.inputs):
                    t.copy_(h, non_blocking=True)
                row.call(stream)
                for h, t in zip(h_out, row.outputs):
                    h.copy_(t, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        e2e_ms = shard.max_over_ranks([e0.elapsed_time(e1)], device=dev)[0]
        line["e2e"] = {"value": round(world * row.units * E / (e2e_ms / 1e3), 2), "unit": unit,
                       "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in row.inputs),
                       "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in row.outputs),
                       "steps": E, "how": "per step: pinned-host -> device copy of the inputs, the call, device -> "
                       "pinned-host copy of the output; the KV cache or the weights stay resident"}
    if world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        cv, sample, times = cpu_op_row(spec, threads, args.cpu_seconds)
        line["cpu_baseline"] = {"value": round(cv, 4), "unit": unit, "cores": threads, "kind": "port",
                                "sample": f"{sample}, {len(times)} repetitions, median taken"}
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- main (ours)

def main() -> int:
    args = parse_args()
    from baremetalinferenceengine_b200.layer import WORKLOADS

    if args.workload in OP_ROWS:
        return run_op_row(args)
    shape = WORKLOADS[args.workload]
    if args.rows:
        shape = shape.with_rows(args.rows)
    if args.impl == "reference":
        return run_reference(args, shape)

    import torch
    import torch.distributed as dist

    from baremetalinferenceengine_b200 import layer, shard

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        log(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 under torchrun")
        return 2
    assert torch.cuda.is_available(), "bench.py needs CUDA devices"
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(values):
        return shard.max_over_ranks(values, device=dev)

    K, W = args.steps, args.warmup
    if W < 3:
        log("warning: fewer than 3 warm-up steps")
    affinity = numa_affinity(dev, local_rank, world)  # before any pinned host allocation
    local, rows = shard.local_shape(shape, rank, world, args.scaling)
    job_bytes = shape.step_bytes() * (world if args.scaling == "weak" else 1)
    job_rows = shape.rows * (world if args.scaling == "weak" else 1)
    log(f"[rank {rank}] allocating {local.name}: tokens [{rows.start}, {rows.stop}) of {job_rows}, "
        f"{local.step_bytes() / 1e9:.2f} GB per step")
    # the same timing branch on every rank: decided by the largest rank's block
    small = shape.with_rows(-(-job_rows // world)).step_bytes() < L2_RESIDENT_BYTES
    # an L2-resident step keeps its inputs and outputs in one arena: its host-buffer
    # (e2e) form is one copy in and one copy out
    b = layer.LayerBuffers(local, dev, seed=1000 + rank, row_offset=rows.start, packed=small)
    stream = torch.cuda.Stream(dev)
    kernels = local.step_kernels()
    nk = len(kernels)

    with torch.cuda.stream(stream):
        for _ in range(W):
            layer.run_step(b, stream)
    stream.synchronize()
    assert b.status.read(stream) == 0, "device status set during warm-up"

    launches = 0
    if not small:
        # Inputs far larger than L2: the step is one CUDA graph (its kernels chained
        # by programmatic dependent launch, no host launch cost between them),
        # replayed K times back to back; each kernel's own duration comes from K more
        # steps launched one kernel at a time with events between the launches.
        step_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(step_graph, stream=stream):
            layer.run_step(b, stream)
        with torch.cuda.stream(stream):
            for _ in range(W):
                step_graph.replay()
        events = [[torch.cuda.Event(enable_timing=True) for _ in range(nk + 1)] for _ in range(K)]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize(dev)
        with ClockSampler(dev) as clocks:
            with torch.cuda.stream(stream):
                start.record(stream)
                for i in range(K):
                    step_graph.replay()
                    launches += nk
                end.record(stream)
            torch.cuda.synchronize(dev)
        barrier()
        elapsed_ms = start.elapsed_time(end)
        for i in range(K):
            layer.run_step(b, stream, events[i])
        torch.cuda.synchronize(dev)
        del step_graph
        per_kernel = [statistics.mean(events[i][j].elapsed_time(events[i][j + 1]) for i in range(K))
                      for j in range(nk)]
    else:
        # An L2-resident working set, where host launch cost would dominate: the
        # step is one CUDA graph, replayed after a 256 MB write that evicts L2 (the
        # timed step is the graph's span); each kernel's own duration comes from a
        # graph of REPEAT back-to-back launches of it (L2 warm), divided by REPEAT.
        repeat = 16
        flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        step_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(step_graph, stream=stream):
            layer.run_step(b)
        kernel_graphs = []
        for _, launch in layer.step_launchers(b):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(repeat):
                    launch()
            kernel_graphs.append(g)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
        kev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(nk)]
               for _ in range(K)]
        with torch.cuda.stream(stream):
            for _ in range(W):
                flush.zero_()
                step_graph.replay()
                for g in kernel_graphs:
                    g.replay()
            barrier()
            torch.cuda.synchronize(dev)
            with ClockSampler(dev) as clocks:
                for i in range(K):
                    flush.zero_()
                    ev[i][0].record(stream)
                    step_graph.replay()
                    ev[i][1].record(stream)
                    launches += nk
                torch.cuda.synchronize(dev)
            for i in range(K):
                for j, g in enumerate(kernel_graphs):
                    kev[i][j][0].record(stream)
                    g.replay()
                    kev[i][j][1].record(stream)
            torch.cuda.synchronize(dev)
        barrier()
        elapsed_ms = sum(e0.elapsed_time(e1) for e0, e1 in ev)
        per_kernel = [statistics.mean(kev[i][j][0].elapsed_time(kev[i][j][1]) for i in range(K)) / repeat
                      for j in range(nk)]
    assert b.status.read(stream) == 0, "device status set during the timed steps"
    res = max_over_ranks([elapsed_ms] + per_kernel)
    elapsed_ms, per_kernel = res[0], res[1:]
    # ---- after the timed region: one more step, its sampled rows checked by the oracle
    parity = None if args.no_parity else sampled_parity(b, stream, rank)
    if parity is not None:
        parity["all_ranks_ok"] = max_over_ranks([0.0 if parity["ok"] else 1.0])[0] == 0.0

    peak, peak_kind = measured_peak()
    value = job_bytes * K / (elapsed_ms / 1e3) / 1e9
    kern = {}
    for (name, nbytes), ms in zip(kernels, per_kernel):
        gbs = nbytes / (ms / 1e3) / 1e9
        kern[name] = {"ms": round(ms, 4), "gb_per_launch": round(nbytes / 1e9, 4), "gbs": round(gbs, 1),
                      "frac": round(gbs / peak, 4)}
    dom_name, dom_bytes = max(kernels, key=lambda kv: kv[1])
    dom_ms = per_kernel[[k for k, _ in kernels].index(dom_name)]
    traffic = load_traffic(shape.name, dom_name)
    roofline = {"kernel": dom_name, "bound": "hbm", "achieved": round(dom_bytes / (dom_ms / 1e3) / 1e9, 1),
                "peak": peak, "unit": "GB/s", "frac": round(dom_bytes / (dom_ms / 1e3) / 1e9 / peak, 4),
                "traffic": traffic, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                if peak_kind == "measured" else "fallback 6650 GB/s",
                "algorithmic_bytes_per_launch": dom_bytes}

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(elapsed_ms / K, 4), "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "bf16" if shape.es == 2 else "f32",
        "data": "synthetic: seeded N(0,1) activations, 1+N(0,0.02) norm weights, N(0,0.02) embeddings",
        "impl": "ours", "config": config_dict(shape, world, args.scaling, local),
        "rows_per_s": round(job_rows * K / (elapsed_ms / 1e3), 1),
        "frac_of_peak": round(value / world / peak, 4),
        "kernels": kern, "roofline": roofline, "gpu_launches": launches,
        "clocks": clocks.summary() if rank == 0 else None,
        "parity_sampled": None if parity is None else parity["all_ranks_ok"],
        "host_affinity": affinity,
    }
    if parity is not None:
        line["parity_detail"] = {k: parity[k] for k in ("rows", "tolerance", "worst_error", "bit_exact", "how")}

    # ---- end to end: inputs from pinned host memory, outputs back, every step
    if not args.no_e2e:
        line["e2e"] = e2e(args, b, local, dev, world, barrier, max_over_ranks)
    # ---- the reference's own CUDA kernels, one token per launch (rank 0, one GPU only)
    if world == 1 and not args.no_ref_gpu:
        del b
        torch.cuda.empty_cache()
        try:
            line["ref_gpu_baseline"] = ref_gpu_baseline(shape, dev, args.ref_gpu_rows, line["rows_per_s"])
        except (OSError, TypeError, ValueError, RuntimeError) as e:  # a baseline leg never sinks the line
            line["ref_gpu_baseline"] = {"unavailable": f"{type(e).__name__}: {e}"}
    # ---- CPU baseline (rank 0, one GPU only)
    if world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        gbs, rows, times, (gbs1, rows1, times1) = cpu_baseline(shape, threads, args.cpu_seconds,
                                                                single_s=min(0.5, args.cpu_seconds))
        line["cpu_baseline"] = {
            "value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{rows} of {shape.rows} tokens of one step (all five ops), oracle_layer_step_mt on "
                      f"{threads} threads, {len(times)} repetitions, {sum(times):.1f} s, median taken"}
        # the reference's loops as written run on one thread: the first rows of the
        # same sample (the per-row estimate comes from a warm probe, so a repetition
        # runs longer than the budget)
        line["cpu_baseline"]["single_thread"] = {
            "value": round(gbs1, 3), "unit": "GB/s", "cores": 1,
            "sample": f"{rows1} tokens, {len(times1)} repetitions, {sum(times1):.1f} s, median taken"}

    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def load_traffic(workload: str, kernel: str):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)[workload][kernel]["dram_bytes_per_launch"]
    except (OSError, KeyError, ValueError, TypeError):
        return None


def numa_affinity(dev, local_rank: int, world: int) -> dict:
    """Binds this process to host CPUs next to its GPU before any pinned host
    memory is allocated, so the pinned pages land on the GPU's NUMA node
    (first touch). Ranks whose GPUs share a CPU list split it evenly. Reads
    sysfs only; returns what it did."""
    import torch

    def gpu_cpus(index):
        props = torch.cuda.get_device_properties(index)
        bus = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        base = f"/sys/bus/pci/devices/{bus}"
        with open(f"{base}/local_cpulist") as f:
            text = f.read().strip()
        try:
            with open(f"{base}/numa_node") as f:
                node = int(f.read().strip())
        except (OSError, ValueError):
            node = -1
        cpus = []
        for part in text.split(","):
            lo, _, hi = part.partition("-")
            cpus.extend(range(int(lo), int(hi or lo) + 1))
        return bus, node, cpus

    try:
        allowed = set(os.sched_getaffinity(0))
        n_local = torch.cuda.device_count()
        lists = [gpu_cpus(i) for i in range(n_local)]
        bus, node, cpus = lists[dev.index]
        sharing = [i for i in range(min(n_local, world)) if lists[i][2] == cpus]
        cpus = [c for c in cpus if c in allowed] or sorted(allowed)
        if dev.index in sharing and len(sharing) > 1:
            k, n = sharing.index(dev.index), len(sharing)
            share = cpus[k * len(cpus) // n:(k + 1) * len(cpus) // n] or cpus
        else:
            share = cpus
        os.sched_setaffinity(0, share)
        return {"gpu_pci": bus, "numa_node": node, "cpus": len(share),
                "cpu_range": f"{min(share)}-{max(share)}", "ranks_sharing_node": len(sharing)}
    except (OSError, ValueError, AttributeError, IndexError, RuntimeError) as e:
        return {"unavailable": f"{type(e).__name__}: {e}"}


def sampled_parity(b, stream, rank: int) -> dict:
    """The oracle as the checker, after the timed region: one more step on the same
    buffers, then the outputs at sampled rows (the first and last, either side of
    every kernel's first grid-stride wrap, the row holding SwiGLU element 2^31, and
    8 seeded rows) compared with the oracle within the stated tolerance."""
    import torch

    from baremetalinferenceengine_b200 import layer
    from oracle import check_step

    sm = torch.cuda.get_device_properties(b.device).multi_processor_count
    rows = check_step.sample_rows(b.shape, sm, random_rows=8, seed=100 + rank)
    sample = check_step.StepSample(b, rows)
    layer.run_step(b, stream)
    stream.synchronize()
    status = b.status.read(stream)
    res = sample.check()
    res["ok"] = bool(res["ok"] and status == 0)
    res["how"] = (f"one untimed step after the timed region; {res['rows']} sampled rows per GPU against the oracle "
                  f"(oracle/check_step.py), worst |got - want| / (1 + |want|) per output")
    return res


def ref_kernels_lib():
    """oracle/_ref/libref_kernels.so with ref_layer_step_rows typed, or None when
    the reference's kernels were not built."""
    from oracle import oracle as orc

    if not os.path.exists(orc.REF_KERNELS_LIB):
        return None
    L = ctypes.CDLL(orc.REF_KERNELS_LIB)
    vp, i64, f32, ci = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
    L.ref_layer_step_rows.restype = i64
    # ops, rows, ids, positions, seq_ids, 16 device buffers, six sizes, theta, eps
    L.ref_layer_step_rows.argtypes = [ci, i64, vp, vp, vp] + [vp] * 16 + [ci] * 6 + [f32, f32]
    return L


def ref_gpu_baseline(shape, dev, max_rows: int, our_rows_per_s: float) -> dict:
    """The reference's own CUDA kernels (src/kernels.cu built for sm_100a into
    oracle/_ref/libref_kernels.so) on this GPU, issued one token at a time as
    ExecutionEngine::run_layers issues them (ref_layer_step_rows): fp32 buffers of
    the workload's dims, the first `max_rows` tokens. Timed with CUDA events on the
    default stream the reference launches on; median of 3 repetitions."""
    import dataclasses

    import torch

    from oracle import oracle as orc

    L = ref_kernels_lib()
    if L is None:
        return {"unavailable": "oracle/_ref/libref_kernels.so is not built (needs the reference's sources)"}
    s32 = dataclasses.replace(shape, dtype=torch.float32)
    n = min(shape.rows, max_rows)
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    rnd = lambda *size: torch.randn(*size, generator=g, device=dev)  # noqa: E731
    ids = torch.randint(0, shape.vocab, (n,), generator=g, device=dev, dtype=torch.int32).cpu()
    if shape.positions == "uniform":
        pos = torch.randint(0, shape.max_seq, (n,), generator=g, device=dev, dtype=torch.int32).cpu()
        seq = (torch.arange(n, dtype=torch.int32) % shape.num_seqs)
    else:
        r = torch.arange(n, dtype=torch.int64)
        pos, seq = (r % shape.max_seq).to(torch.int32), (r // shape.max_seq).to(torch.int32)
    nseq = int(seq.max()) + 1
    D, F = shape.dim, shape.ffn
    t = {"embed": rnd(shape.vocab, D) * 0.02, "hidden": torch.empty(n, D, device=dev), "attn_out": rnd(n, D),
         "w_attn": rnd(D) * 0.02 + 1, "y_attn": torch.empty(n, D, device=dev), "q": rnd(n, shape.hq, shape.hd),
         "k": rnd(n, shape.hkv, shape.hd), "v": rnd(n, shape.hkv, shape.hd),
         "k_cache": torch.zeros(nseq, shape.hkv, shape.max_seq, shape.hd, device=dev),
         "v_cache": torch.zeros(nseq, shape.hkv, shape.max_seq, shape.hd, device=dev), "ffn_out": rnd(n, D),
         "w_ffn": rnd(D) * 0.02 + 1, "y_ffn": torch.empty(n, D, device=dev), "gate": rnd(n, F), "up": rnd(n, F),
         "act": torch.empty(n, F, device=dev)}
    order = ["embed", "hidden", "attn_out", "w_attn", "y_attn", "q", "k", "v", "k_cache", "v_cache", "ffn_out",
             "w_ffn", "y_ffn", "gate", "up", "act"]
    ptrs = [t[k].data_ptr() for k in order]
    default = torch.cuda.default_stream(dev)
    torch.cuda.synchronize(dev)

    def run(ops):
        return L.ref_layer_step_rows(ops, n, ids.data_ptr(), pos.data_ptr(), seq.data_ptr(), *ptrs, D, shape.hq,
                                     shape.hkv, shape.hd, F, shape.max_seq, shape.theta, shape.eps)

    def timed(ops):
        run(ops)  # warm
        ms = []
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(default)
            issued = run(ops)
            e1.record(default)
            torch.cuda.synchronize(dev)
            ms.append(e0.elapsed_time(e1))
        return statistics.median(ms), issued

    per_row = s32.bytes_per_row()
    op_bits = {"embed_gather": (1, per_row["embed_gather"]), "add_rmsnorm_attn": (2, per_row["add_rmsnorm"]),
               "rope_kv_store": (4, per_row["rope_kv_store"]), "add_rmsnorm_ffn": (8, per_row["add_rmsnorm"]),
               "swiglu": (16, per_row["swiglu"])}
    if shape.kind == "stress":
        op_bits = {k: op_bits[k] for k in ("embed_gather", "swiglu")}
    per_op = {}
    for name, (bit, nbytes) in op_bits.items():
        ms, _ = timed(bit)
        per_op[name] = {"rows_per_s": round(n / (ms / 1e3), 1), "gbs": round(nbytes * n / (ms / 1e3) / 1e9, 2),
                        "us_per_row": round(ms * 1e3 / n, 2)}
    all_ops = sum(bit for bit, _ in op_bits.values())
    ms, issued = timed(all_ops)
    step_bytes = sum(nb for _, nb in op_bits.values()) * n
    rows_per_s = n / (ms / 1e3)
    del t
    torch.cuda.empty_cache()
    return {"value": round(step_bytes / (ms / 1e3) / 1e9, 3), "unit": "GB/s", "rows_per_s": round(rows_per_s, 1),
            "dtype": "f32", "launches_per_row": issued // n, "per_op": per_op,
            "ours_over_reference_rows_per_s": round(our_rows_per_s / rows_per_s, 1),
            "kind": "reference CUDA kernels (src/kernels.cu, sm_100a), one token per launch as "
                    "ExecutionEngine::run_layers issues them",
            "sample": f"the first {n} of {shape.rows} tokens of {shape.name} at its dims in fp32 (the reference's "
                      f"kernels are fp32 only; ours run {('bf16' if shape.es == 2 else 'f32')}), CUDA events on "
                      f"the default stream, median of 3"}


def pcie_link(dev, h2d, d2h, barrier, max_over_ranks, world: int, nbytes: int = 1 << 30, reps: int = 3,
              mix=None) -> dict:
    """Host<->device bandwidth of pinned copies, the roofline of the e2e leg: H2D
    alone, D2H alone, and both directions at once on two streams. Every rank
    copies at the same time (a barrier before each phase), so the per-GPU rates
    are those each GPU gets while all N copy: the host side is shared.
    mix = (h2d_bytes, d2h_bytes) of one step adds a fourth phase, both directions
    at once in that ratio (the larger side nbytes): the time the link needs for
    the step's own copies, with nothing else running."""
    import torch

    host_a = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    host_b = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dev_a = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    dev_b = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    def timed(streams_ops):
        barrier()
        torch.cuda.synchronize(dev)
        evs = []
        for st, op in streams_ops:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(st):
                e0.record(st)
                for _ in range(reps):
                    op()
                e1.record(st)
            evs.append((e0, e1))
        torch.cuda.synchronize(dev)
        own = max(e0.elapsed_time(e1) for e0, e1 in evs) / 1e3
        return own, max_over_ranks([own])[0]

    up = lambda: dev_a.copy_(host_a, non_blocking=True)  # noqa: E731
    down = lambda: host_b.copy_(dev_b, non_blocking=True)  # noqa: E731
    timed([(h2d, up), (d2h, down)])  # warm
    t_up, t_up_all = timed([(h2d, up)])
    t_down, t_down_all = timed([(d2h, down)])
    t_both, t_both_all = timed([(h2d, up), (d2h, down)])
    gb = nbytes * reps / 1e9
    out = {"h2d_gbs": round(gb / t_up, 1), "d2h_gbs": round(gb / t_down, 1),
           "bidirectional_gbs": round(2 * gb / t_both, 1),
           "aggregate": {"h2d_gbs": round(world * gb / t_up_all, 1), "d2h_gbs": round(world * gb / t_down_all, 1),
                         "bidirectional_gbs": round(2 * world * gb / t_both_all, 1), "gpus": world},
           "how": f"pinned 1 GiB copies x{reps} per GPU, all {world} GPU(s) at once, CUDA events; per-GPU rates "
                  f"are this GPU's own, aggregate = all GPUs' bytes / the slowest GPU's time"}
    if mix is not None and max(mix) > 0:
        scale = nbytes / max(mix)
        n_up, n_down = (min(nbytes, int(x * scale)) // 512 * 512 for x in mix)
        up_mix = lambda: dev_a[:n_up].copy_(host_a[:n_up], non_blocking=True)  # noqa: E731
        down_mix = lambda: host_b[:n_down].copy_(dev_b[:n_down], non_blocking=True)  # noqa: E731
        _, t_mix_all = timed([(h2d, up_mix), (d2h, down_mix)])
        # seconds the link needs for one step's copies (every GPU copying its own at once)
        out["step_mix"] = {"h2d_bytes": n_up, "d2h_bytes": n_down, "s_per_step": t_mix_all / reps / scale,
                           "how": "H2D and D2H at once in the step's byte ratio, all GPUs at once, scaled to "
                                  "one step's bytes; the slowest GPU's time"}
    del host_a, host_b, dev_a, dev_b
    return out


def bytes_per_row(b, names) -> float:
    return b.nbytes(names) / b.shape.rows


def e2e(args, b, shape, dev, world, barrier, max_over_ranks):
    """The same step through the public API with host buffers: every step copies
    its inputs in from pinned host memory and its outputs back, chunked over rows
    so copies in both directions overlap the kernels of other chunks, and the
    next step's first chunks come in while this step's last chunks go out. Its
    roofline is the host link measured with every GPU copying at once: a step
    cannot end before its H2D bytes, its D2H bytes and their sum have crossed at
    the measured H2D, D2H and bidirectional rates."""
    import torch

    from baremetalinferenceengine_b200 import layer

    names_in, names_out = b.inputs(), b.outputs()
    io_per_row = (b.nbytes(names_in) + b.nbytes(names_out)) / shape.rows
    try:
        import psutil

        avail = psutil.virtual_memory().available
    except ImportError:
        avail = 0
    # Every rank pins its own host buffers; all ranks together stay under 40% of
    # the host's free memory. The step then covers the first R rows that fit
    # (throughput in GB/s does not depend on R once R is thousands of tokens).
    R = int(min(shape.rows, 0.4 * avail / world // io_per_row))
    R = int(-max_over_ranks([-R])[0])  # the same rows (and the same branch) on every rank
    if R < min(shape.rows, 1024):
        return {"unavailable": f"host has {avail / 1e9:.1f} GB free: too little to pin a step's buffers"}
    # A step that fits in L2 is a decode-sized batch: one copy in, one launch
    # sequence, one copy out, repeated enough times to time.
    small = shape.step_bytes() < L2_RESIDENT_BYTES

    def pinned(t):
        return torch.empty((R,) + tuple(t.shape[1:]), dtype=t.dtype, device="cpu", pin_memory=True)

    h2d, comp, d2h = (torch.cuda.Stream(dev) for _ in range(3))
    chunks = 1 if small else max(1, min(args.e2e_chunks, R))
    size = math.ceil(R / chunks)
    slices = [slice(i, min(R, i + size)) for i in range(0, R, size)]
    arena = small and b.arena is not None and R == shape.rows
    if arena:
        # one copy in (every input, q included) and one copy out (q and every output),
        # alternating between two arenas so a step's outputs go back while the next
        # step's inputs come in
        h_arena_in = torch.empty(b.in_end, dtype=torch.uint8, pin_memory=True)
        h_arena_out = [torch.empty(b.arena.numel() - b.out_start, dtype=torch.uint8, pin_memory=True)
                       for _ in range(2)]
        h_arena_in.copy_(b.arena[:b.in_end])
        bufs = [b, b.with_arena(torch.empty_like(b.arena))]
        free = [torch.cuda.Event(), torch.cuda.Event()]
        parity = [0]
    else:
        h_in = {n: pinned(getattr(b, n)) for n in names_in}
        h_out = {n: pinned(getattr(b, n)) for n in names_out}
        for n in names_in:
            h_in[n].copy_(getattr(b, n)[:R])

    def step_arena():
        x = parity[0]
        parity[0] ^= 1
        bx = bufs[x]
        h2d.wait_event(free[x])  # the step two back, on this arena, has been copied out
        ev_in, ev_k = torch.cuda.Event(), torch.cuda.Event()
        with torch.cuda.stream(h2d):
            bx.arena[:b.in_end].copy_(h_arena_in, non_blocking=True)
            ev_in.record(h2d)
        comp.wait_event(ev_in)
        with torch.cuda.stream(comp):
            layer.run_step(bx, comp)
            ev_k.record(comp)
        d2h.wait_event(ev_k)
        with torch.cuda.stream(d2h):
            h_arena_out[x].copy_(bx.arena[b.out_start:], non_blocking=True)
            free[x].record(d2h)

    # chunk_out[j]: the last D2H of chunk j's rows. The next step's H2D into those
    # rows waits for it (its inputs were consumed by then and q, an input updated
    # in place, has been read back), so the next step's first chunks come in while
    # this step's last chunks go out.
    chunk_out = [torch.cuda.Event() for _ in slices]

    def step():
        if arena:
            return step_arena()
        for sl, out_ev in zip(slices, chunk_out):
            ev_in, ev_k = torch.cuda.Event(), torch.cuda.Event()
            h2d.wait_event(out_ev)
            with torch.cuda.stream(h2d):
                for n in names_in:
                    getattr(b, n)[sl].copy_(h_in[n][sl], non_blocking=True)
                ev_in.record(h2d)
            comp.wait_event(ev_in)
            with torch.cuda.stream(comp):
                layer.run_step(b, comp, rows=sl)
                ev_k.record(comp)
            d2h.wait_event(ev_k)
            with torch.cuda.stream(d2h):
                for n in names_out:
                    h_out[n][sl].copy_(getattr(b, n)[sl], non_blocking=True)
                out_ev.record(d2h)

    for _ in range(2):
        step()
    torch.cuda.synchronize(dev)
    E = max(50 if small else 1, args.e2e_steps)
    barrier()
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(h2d)
    comp.wait_event(t0)
    d2h.wait_event(t0)
    for _ in range(E):
        step()
    t1.record(d2h)
    torch.cuda.synchronize(dev)
    barrier()
    ms = max_over_ranks([t0.elapsed_time(t1)])[0]
    if arena:
        bin_, bout = b.in_end, b.arena.numel() - b.out_start
        del h_arena_in, h_arena_out
    else:
        bin_, bout = bytes_per_row(b, names_in) * R, bytes_per_row(b, names_out) * R
        del h_in, h_out
    link = pcie_link(dev, h2d, d2h, barrier, max_over_ranks, world, mix=(bin_, bout))
    step_bytes = shape.with_rows(R).step_bytes()
    gbs = world * step_bytes * E / (ms / 1e3) / 1e9
    h2d_rate = bin_ / (ms / E / 1e3) / 1e9
    # host-side lower bound of one step on this GPU while every GPU copies, then the
    # job's: each direction at its own rate, both at the bidirectional rate, and the
    # step's own mix of copies timed alone
    t_link = max(bin_ / (link["h2d_gbs"] * 1e9), bout / (link["d2h_gbs"] * 1e9),
                 (bin_ + bout) / (link["bidirectional_gbs"] * 1e9), link["step_mix"]["s_per_step"])
    t_link = max_over_ranks([t_link])[0]
    roof = world * step_bytes / t_link / 1e9
    return {"value": round(gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": int(bin_), "d2h_bytes_per_step": int(bout),
            "rows_per_step": R, "steps": E, "ms_per_step": round(ms / E, 4), "chunks": len(slices),
            "link": link, "h2d_gbs_achieved": round(h2d_rate, 1),
            "host_gbs_achieved": round(world * (bin_ + bout) / (ms / E / 1e3) / 1e9, 1),
            "roofline": {"gbs": round(roof, 2), "ms_per_step": round(t_link * 1e3, 3),
                         "how": "max over GPUs of max(H2D bytes / H2D rate, D2H bytes / D2H rate, both / "
                                "bidirectional rate, the time of the step's H2D and D2H bytes copied at once "
                                "with nothing else running), all measured with every GPU copying at once"},
            "frac_of_link": round(gbs / roof, 3),
            "copies": "one H2D copy of the step's input arena and one D2H copy of its output arena" if arena else
                      f"one copy per tensor and chunk ({len(slices)} chunks over rows)",
            "how": "per step: pinned-host -> device copies of every input, the step's kernels, device -> pinned-host "
                   "copies of every output, on three streams (chunks overlap copies and kernels, and a step's first "
                   "chunks come in while the previous step's last chunks go out); CUDA events, max over ranks; "
                   "host buffers pinned after binding the rank to its GPU's NUMA-local CPUs"}


if __name__ == "__main__":
    sys.exit(main())

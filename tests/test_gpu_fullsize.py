"""Parity at the benchmarked sizes: one whole layer step of each large workload.

The step runs through the C ABI exactly as bench.py runs it (layer.run_step on
layer.LayerBuffers): Llama-3-70B (131072 tokens, dim 8192, FFN 28672: the
SwiGLU spans 3.76e9 elements, past 2^31), Llama-3-8B prefill (32768 tokens)
and the SwiGLU stress workload (65536 Zipf(1.1) ids, 65536 x 14336 with 1% of
gate/up at +-20). Two checks per workload:

1. Sampled rows against the oracle (oracle/check_step.py): the first and last
   row, the rows on either side of every kernel's first grid-stride wrap, the
   row holding SwiGLU element 2^31, and a seeded spread; bf16 within 1e-2 in the
   reference's metric |got - want| / (1 + |want|) (tests/kernel_tests.cu:40),
   the residual and the V cache slots bit-exact.
2. Every row against a PyTorch fp32/fp64 restatement of the same ops on the
   GPU, chunk by chunk: the residual (gather + two fp32 adds, each rounded once)
   bit-exact, the norms, RoPE (Q in place, K into its cache slot) and SwiGLU
   within the same tolerance, V slots bit-exact. A kernel that skipped rows
   on a later trip fails here whatever the sample.
"""
import math

import pytest
import torch

from baremetalinferenceengine_b200 import layer
from oracle import check_step

pytestmark = pytest.mark.gpu

WORKLOADS = ["llama70b_bf16", "llama8b_prefill_bf16", "swiglu_stress_bf16"]
CHUNK = 8192  # rows per chunk of the all-rows check
TOL = {2: 1e-2, 4: 1e-5}


def metric(got: torch.Tensor, want: torch.Tensor) -> float:
    """max |got - want| / (1 + |want|) on the device, NaN counted as a failure."""
    w = want.double()
    err = (got.double() - w).abs() / (1.0 + w.abs())
    if torch.isnan(err).any():
        return math.inf
    return float(err.max()) if err.numel() else 0.0


def rope_ref(x: torch.Tensor, pos: torch.Tensor, theta: float) -> torch.Tensor:
    """Half-split RoPE in fp64 (the angle of tests/kernel_tests.cu:180): x [n, heads, hd]."""
    hd = x.shape[-1]
    half = hd // 2
    i = torch.arange(half, device=x.device, dtype=torch.float64)
    ang = pos.double()[:, None] / torch.pow(torch.tensor(theta, dtype=torch.float64, device=x.device), 2.0 * i / hd)
    c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    xd = x.double()
    a, b = xd[..., :half], xd[..., half:]
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1)


def rmsnorm_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def check_all_rows(b, q_before) -> dict:
    s = b.shape
    tol = TOL[s.es]
    worst = {}
    exact = {"hidden": True, "v_cache": True}

    def note(name, err):
        worst[name] = max(worst.get(name, 0.0), err)

    for r0 in range(0, s.rows, CHUNK):
        sl = slice(r0, min(s.rows, r0 + CHUNK))
        h0 = b.embed.index_select(0, b.ids[sl].long())
        if s.kind == "stress":
            exact["hidden"] &= torch.equal(b.hidden[sl].view(torch.int16), h0.view(torch.int16))
        else:
            h1 = (h0.float() + b.attn_out[sl].float()).to(s.dtype)
            h2 = (h1.float() + b.ffn_out[sl].float()).to(s.dtype)
            iv = torch.int32 if s.es == 4 else torch.int16
            exact["hidden"] &= torch.equal(b.hidden[sl].view(iv), h2.view(iv))
            note("y_attn", metric(b.y_attn[sl], rmsnorm_ref(h1, b.w_attn, s.eps)))
            note("y_ffn", metric(b.y_ffn[sl], rmsnorm_ref(h2, b.w_ffn, s.eps)))
            pos = b.positions[sl].long()
            note("q", metric(b.q[sl], rope_ref(q_before[sl], pos, s.theta)))
            seq = b.seq_ids[sl].long()
            note("k_cache", metric(b.k_cache[seq, :, pos, :], rope_ref(b.k[sl], pos, s.theta)))
            exact["v_cache"] &= torch.equal(b.v_cache[seq, :, pos, :].view(torch.int16), b.v[sl].view(torch.int16))
        g, u = b.gate[sl].float(), b.up[sl].float()
        note("act", metric(b.act[sl], g / (1.0 + torch.exp(-g)) * u))
    if s.kind == "stress":
        del exact["v_cache"]
    return {"worst": worst, "exact": exact, "ok": all(v <= tol for v in worst.values()) and all(exact.values())}


@pytest.mark.parametrize("name", WORKLOADS)
def test_full_size_step(cuda, name):
    shape = layer.WORKLOADS[name]
    torch.cuda.empty_cache()
    b = layer.LayerBuffers(shape, cuda, seed=31)
    if shape.positions == "tiled" and shape.kind == "layer":
        # every (sequence, position) cache slot is written by exactly one token
        assert shape.rows <= shape.num_seqs * shape.max_seq
    sm = torch.cuda.get_device_properties(cuda).multi_processor_count
    rows = check_step.sample_rows(shape, sm, random_rows=48, seed=5)
    wraps = check_step.wrap_rows(shape, sm)
    for kernel, r in wraps.items():
        if r is not None:
            assert r in rows and r - 1 in rows, (kernel, r)
    sample = check_step.StepSample(b, rows)
    q_before = b.q.clone() if shape.kind == "layer" else None
    launches = layer.run_step(b)
    torch.cuda.synchronize(cuda)
    assert launches == len(shape.step_kernels())
    assert b.status.read() == 0

    res = sample.check()
    assert res["ok"], res
    full = check_all_rows(b, q_before)
    assert full["ok"], full
    del b, q_before, sample
    torch.cuda.empty_cache()


"""The full-size step checker (oracle/check_step.py), on the CPU.

The sampled-row checker must pass a step whose outputs are the oracle's own and
fail one with a planted mistake (the mistake is planted in CPU tensors; no GPU
runs). The grid-stride wrap rows it samples are pinned for the 70B step on 148
SMs.
"""
import dataclasses

import numpy as np
import torch

from baremetalinferenceengine_b200 import layer
from oracle import check_step
from oracle import oracle as orc
from tests.helpers import from_np, to_np

TINY = layer.LayerShape("tiny_bf16", rows=64, dim=64, hq=4, hkv=2, hd=16, ffn=96, vocab=50, theta=1e4, max_seq=32,
                        num_seqs=2, dtype=torch.bfloat16)


def oracle_step(b, q_before):
    """Writes the oracle's outputs of one step into b's (CPU) tensors."""
    s = b.shape
    h0, bad = orc.gather(to_np(b.embed), to_np(b.ids))
    assert bad == 0
    h1, y_attn = orc.add_rmsnorm(h0, to_np(b.attn_out), to_np(b.w_attn), s.eps)
    q, kc, vc, bad = orc.rope_kv_store(to_np(q_before), to_np(b.k), to_np(b.v), to_np(b.positions),
                                       to_np(b.k_cache), to_np(b.v_cache), s.theta, seq_ids=to_np(b.seq_ids))
    assert bad == 0
    h2, y_ffn = orc.add_rmsnorm(h1, to_np(b.ffn_out), to_np(b.w_ffn), s.eps)
    for name, arr in (("hidden", h2), ("y_attn", y_attn), ("q", q), ("k_cache", kc), ("v_cache", vc),
                      ("y_ffn", y_ffn), ("act", orc.swiglu(to_np(b.gate), to_np(b.up)))):
        getattr(b, name).copy_(from_np(arr).view(getattr(b, name).shape))


def test_checker_passes_the_oracle_and_catches_planted_mistakes():
    b = layer.LayerBuffers(TINY, "cpu", seed=3, with_table=False)
    rows = check_step.sample_rows(TINY, sm_count=1, random_rows=8, seed=1)
    sample = check_step.StepSample(b, rows)
    q_before = b.q.clone()
    oracle_step(b, q_before)
    res = sample.check()
    assert res["ok"], res
    assert set(res["worst_error"]) == {"y_attn", "y_ffn", "q", "k_cache", "act"}
    assert res["bit_exact"] == {"hidden": True, "v_cache": True}

    r = int(rows[len(rows) // 2])
    b.act[r, 5] = b.act[r, 5] * 1.5 + 1.0  # a wrong SwiGLU value at a sampled row
    assert not sample.check()["ok"]
    oracle_step(b, q_before)
    h = b.hidden.view(torch.int16)
    h[r, 0] ^= 1  # one ulp off in the residual: bit-exactness is required
    res = sample.check()
    assert not res["ok"] and res["bit_exact"]["hidden"] is False
    oracle_step(b, q_before)
    pos, seq = int(b.positions[r]), int(b.seq_ids[r])
    b.k_cache[seq, 1, pos, 3] += 0.5  # a wrong K cache slot
    assert not sample.check()["ok"]


def test_wrap_rows_of_the_70b_step_on_148_sms():
    """The 70B step (131072 x 8192 bf16, FFN 28672): gather and both norms wrap at
    row 75776, RoPE at 18944 tokens, SwiGLU's second trip starts inside row 5412;
    flat element 2^31 of gate/up lies in row 74898."""
    shape = layer.WORKLOADS["llama70b_bf16"]
    assert check_step.wrap_rows(shape, 148) == {"embed_gather": 75776, "add_rmsnorm": 75776,
                                                 "rope_kv_store": 18944, "swiglu": 5412}
    rows = check_step.sample_rows(shape, 148)
    for r in (0, 131071, 75775, 75776, 18943, 18944, 5412, 5413, 74898):
        assert r in rows
    assert np.all(np.diff(rows) > 0)
    # a rank's own rows only
    assert check_step.sample_rows(shape, 148, limit=16384).max() == 16383


def test_wrap_rows_other_workloads():
    w = check_step.wrap_rows(layer.WORKLOADS["llama8b_prefill_bf16"], 148)
    assert w["add_rmsnorm"] is None and w["embed_gather"] is None  # 2 rows a block: one trip covers 32768
    assert w["rope_kv_store"] == 18944
    stress = check_step.wrap_rows(layer.WORKLOADS["swiglu_stress_bf16"], 148)
    assert stress["rope_kv_store"] is None and stress["swiglu"] == 155189248 // 14336
    small = dataclasses.replace(layer.WORKLOADS["llama8b_decode_bf16"])
    assert all(v is None for v in check_step.wrap_rows(small, 148).values())

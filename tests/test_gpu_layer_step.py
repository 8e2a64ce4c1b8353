"""The layer step entry point (bm_layer_step) against the oracle, on the GPU.

Decode-sized batches (at most 512 tokens) run as one launch holding row jobs
(gather, both residual adds and norms), token jobs (RoPE + K/V) and SwiGLU jobs;
larger batches issue the five batched kernels. Both forms are checked against
the oracle (the reference's double-precision check loops, tests/kernel_tests.cu:
75-79, 122, 175-187, 206, 223-226, and the row copy of
src/execution_engine.cu:98-99): fp32 within 1e-5 and bf16 within 1e-2 in the
reference's metric |got - want| / (1 + |want|), the residual and the cache
copies bit-exact. The single launch is also compared with the five separate
calls on the same inputs: everything but the norms bit for bit (the norms sum
in another order), and bad ids / positions / sequences behave the same way.
"""
import dataclasses

import numpy as np
import pytest
import torch

from baremetalinferenceengine_b200 import _lib, layer, ops
from oracle import oracle as orc
from tests.helpers import TOL, bits_equal, to_np

pytestmark = pytest.mark.gpu

W = layer.WORKLOADS
SHAPES = {
    "tinyllama_fp32": W["tinyllama_fp32"],
    "llama8b_decode_bf16": W["llama8b_decode_bf16"],
    "llama8b_decode_fp32": W["llama8b_decode_fp32"],
    "llama70b_96_bf16": W["llama70b_bf16"].with_rows(96),
    "llama70b_96_fp32": dataclasses.replace(W["llama70b_bf16"].with_rows(96), dtype=torch.float32),
    "llama8b_512_bf16": W["llama8b_prefill_bf16"].with_rows(512),   # the largest single launch
    "llama8b_513_bf16": W["llama8b_prefill_bf16"].with_rows(513),   # the first five-kernel batch
}


def small(shape, cuda, seed=3):
    """Buffers of `shape` with the embedding table and caches cut to what the rows
    use (a full 128256-row table and 64 sequences of cache are GBs; the kernel
    sees the same layout). Decode-shaped batches get distinct positions over 4
    sequences, so no two tokens write one cache slot."""
    tiled = shape.positions == "tiled"
    s = dataclasses.replace(shape, vocab=min(shape.vocab, 4096),
                            num_seqs=-(-shape.rows // shape.max_seq) if tiled else min(shape.num_seqs, 4))
    b = layer.LayerBuffers(s, cuda, seed=seed)
    if not tiled:
        r = torch.arange(s.rows, dtype=torch.int64, device=cuda)
        b.positions.copy_((r * 997 + 13) % s.max_seq)
        b.seq_ids.copy_(r % s.num_seqs)
    return b


def call_step(b, table=True, status=None):
    s = b.shape
    ops.layer_step(b.ids, b.embed, b.hidden, b.attn_out, b.w_attn, b.y_attn, b.q, b.k, b.v, b.positions, b.k_cache,
                   b.v_cache, b.ffn_out, b.w_ffn, b.y_ffn, b.gate, b.up, b.act, s.eps,
                   table=b.table if table else None, theta=s.theta, seq_ids=b.seq_ids,
                   status=status if status is not None else b.status)


def separate(b, table=True, status=None):
    s = b.shape
    st = status if status is not None else b.status
    ops.embed_gather(b.embed, b.ids, out=b.hidden, status=st)
    ops.add_rmsnorm(b.hidden, b.attn_out, b.w_attn, s.eps, out=b.y_attn)
    ops.rope_kv_store(b.q, b.k, b.v, b.positions, b.k_cache, b.v_cache, table=b.table if table else None,
                      theta=s.theta, seq_ids=b.seq_ids, status=st)
    ops.add_rmsnorm(b.hidden, b.ffn_out, b.w_ffn, s.eps, out=b.y_ffn)
    ops.swiglu(b.gate, b.up, out=b.act)


def oracle_step(host, s):
    h0, bad_id = orc.gather(host["embed"], host["ids"])
    h1, y_attn = orc.add_rmsnorm(h0, host["attn_out"], host["w_attn"], s.eps)
    q, kc, vc, bad_pos = orc.rope_kv_store(host["q"], host["k"], host["v"], host["positions"], host["k_cache"],
                                           host["v_cache"], s.theta, seq_ids=host["seq_ids"])
    h2, y_ffn = orc.add_rmsnorm(h1, host["ffn_out"], host["w_ffn"], s.eps)
    return {"hidden": h2, "y_attn": y_attn, "q": q, "k_cache": kc, "v_cache": vc, "y_ffn": y_ffn,
            "act": orc.swiglu(host["gate"], host["up"])}, bad_id | bad_pos


INPUTS = ("embed", "ids", "attn_out", "w_attn", "q", "k", "v", "positions", "seq_ids", "k_cache", "v_cache",
          "ffn_out", "w_ffn", "gate", "up")
EXACT = ("hidden", "v_cache")


def snapshot(b):
    return {n: to_np(getattr(b, n)) for n in INPUTS}


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("table", [True, False], ids=["table", "fp64"])
def test_layer_step_matches_the_oracle(cuda, name, table):
    shape = SHAPES[name]
    b = small(shape, cuda)
    host = snapshot(b)
    call_step(b, table=table)
    torch.cuda.synchronize(cuda)
    assert b.status.read() == 0
    want, bad = oracle_step(host, b.shape)
    assert bad == 0
    tol = TOL[shape.dtype]
    for n, w in want.items():
        got = to_np(getattr(b, n))
        if n in EXACT:
            assert np.array_equal(got.reshape(w.shape), w), n
        else:
            assert orc.worst_error(got, w) <= tol, n


@pytest.mark.parametrize("name", ["tinyllama_fp32", "llama8b_decode_bf16", "llama70b_96_fp32"])
def test_single_launch_equals_the_five_calls(cuda, name):
    shape = SHAPES[name]
    a, c = small(shape, cuda, seed=9), small(shape, cuda, seed=9)
    call_step(a)
    separate(c)
    torch.cuda.synchronize(cuda)
    assert a.status.read() == 0 and c.status.read() == 0
    for n in ("hidden", "q", "k_cache", "v_cache", "act"):
        assert bits_equal(getattr(a, n), getattr(c, n)), n
    for n in ("y_attn", "y_ffn"):
        assert orc.worst_error(to_np(getattr(a, n)), to_np(getattr(c, n))) <= TOL[shape.dtype], n


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_bad_rows_flag_and_skip_like_the_five_calls(cuda, dt):
    """A bad id leaves hidden's old row as the gather does (the adds still run on
    it); a bad position or sequence skips that token's RoPE and cache writes."""
    shape = dataclasses.replace(SHAPES["llama8b_decode_bf16"], dtype=dt)
    a, c = small(shape, cuda, seed=4), small(shape, cuda, seed=4)
    for b in (a, c):
        b.hidden.fill_(0.25)
        b.ids[3] = -1
        b.ids[10] = b.shape.vocab
        b.positions[5] = b.shape.max_seq
        b.seq_ids[7] = b.shape.num_seqs
    sa, sc = ops.DeviceStatus(cuda), ops.DeviceStatus(cuda)
    call_step(a, status=sa)
    separate(c, status=sc)
    want = _lib.BM_DEVERR_BAD_ID | _lib.BM_DEVERR_BAD_POSITION | _lib.BM_DEVERR_BAD_SEQUENCE
    assert sa.read() == want and sc.read() == want
    for n in ("hidden", "q", "k_cache", "v_cache", "act"):
        assert bits_equal(getattr(a, n), getattr(c, n)), n
    for n in ("y_attn", "y_ffn"):
        assert orc.worst_error(to_np(getattr(a, n)), to_np(getattr(c, n))) <= TOL[dt], n


def test_unaligned_or_ragged_steps_take_the_five_kernels(cuda):
    """dim 301 has no whole 16-byte vectors: the step issues the five kernels and
    still matches the oracle."""
    shape = layer.LayerShape("ragged", rows=17, dim=301, hq=4, hkv=2, hd=12, ffn=77, vocab=50, theta=1e4,
                             max_seq=32, num_seqs=1, dtype=torch.float32)
    b = layer.LayerBuffers(shape, cuda, seed=2)
    host = snapshot(b)
    call_step(b)
    torch.cuda.synchronize(cuda)
    assert b.status.read() == 0
    want, _ = oracle_step(host, shape)
    for n, w in want.items():
        got = to_np(getattr(b, n))
        if n in EXACT:
            assert np.array_equal(got.reshape(w.shape), w), n
        else:
            assert orc.worst_error(got, w) <= TOL[torch.float32], n


"""bm_rope_kv_decode_attention: the new token's RoPE + K/V store and decode attention
in one call, against the two calls it replaces and against the oracle.

The two calls are bm_rope_kv_store then bm_decode_attention (the engine's order,
src/execution_engine.cu:113-116). On the CUDA-core path the fused launch uses
their arithmetic, so the output and both caches are compared bit for bit; the
oracle (the reference's RoPE and attention check loops, tests/kernel_tests.cu:
175-187, 229-258, in double precision) bounds both: fp32 within 1e-5, bf16 within
1e-2 in the reference's metric.
"""
import ctypes

import pytest
import torch

from baremetalinferenceengine_b200 import _lib, ops
from oracle import oracle as orc
from tests.helpers import TOL, bits_equal, from_np, gen, randn, to_np
from tests.test_gpu_attention import oracle_attention

pytestmark = pytest.mark.gpu

THETA = 10000.0


def case(cuda, dt, batch, hq, hkv, hd, max_seq, num_seqs, seed, pos_mode="last"):
    g = gen(seed)
    q = randn((batch, hq, hd), dt, g)
    k = randn((batch, hkv, hd), dt, g)
    v = randn((batch, hkv, hd), dt, g)
    kc = randn((num_seqs, hkv, max_seq, hd), dt, g)
    vc = randn((num_seqs, hkv, max_seq, hd), dt, g)
    seq_ids = torch.randperm(num_seqs, generator=g)[:batch].to(torch.int32)  # one query per sequence
    lens = torch.randint(1, max_seq + 1, (batch,), generator=g, dtype=torch.int32)
    lens[0] = max_seq
    if pos_mode == "last":
        positions = lens - 1
    else:  # anywhere before the end of the attended range
        positions = (torch.rand(batch, generator=g) * lens.to(torch.float32)).to(torch.int32).clamp(max=max_seq - 1)
    return dict(q=q, k=k, v=v, kc=kc, vc=vc, seq_ids=seq_ids, lens=lens, positions=positions)


def call_fused(cuda, c, table, max_len, status, workspace=True):
    L = _lib.load()
    batch, hq, hd = c["q"].shape
    num_seqs, hkv, max_seq, _ = c["kc"].shape
    need = ctypes.c_size_t()
    _lib.check(L.bm_decode_attention_workspace_size(batch, hq, hkv, hd, max_len, ctypes.byref(need)))
    ws = torch.empty(max(need.value, 1), dtype=torch.uint8, device=cuda) if workspace else None
    d = {n: c[n].to(cuda) for n in ("q", "k", "v", "kc", "vc", "seq_ids", "lens", "positions")}
    out = torch.full((batch, hq, hd), 7.0, dtype=c["q"].dtype, device=cuda)
    _lib.check(L.bm_rope_kv_decode_attention(
        out.data_ptr(), d["q"].data_ptr(), d["k"].data_ptr(), d["v"].data_ptr(), d["positions"].data_ptr(), table.ptr,
        table.max_pos, d["seq_ids"].data_ptr(), d["kc"].data_ptr(), d["vc"].data_ptr(), d["lens"].data_ptr(), max_len,
        batch, hq, hkv, hd, max_seq, num_seqs, 0.0, None if ws is None else ws.data_ptr(),
        need.value if ws is not None else 0, ops.bm_dtype(c["q"]), status.ptr, torch.cuda.current_stream(cuda).cuda_stream))
    return out, d["kc"], d["vc"]


def call_unfused(cuda, c, table, max_len, status, workspace=True):
    L = _lib.load()
    batch, hq, hd = c["q"].shape
    num_seqs, hkv, max_seq, _ = c["kc"].shape
    d = {n: c[n].to(cuda) for n in ("q", "k", "v", "kc", "vc", "seq_ids", "lens", "positions")}
    ops.rope_kv_store(d["q"], d["k"], d["v"], d["positions"], d["kc"], d["vc"], table=table, seq_ids=d["seq_ids"],
                      status=status)
    need = ctypes.c_size_t()
    _lib.check(L.bm_decode_attention_workspace_size(batch, hq, hkv, hd, max_len, ctypes.byref(need)))
    ws = torch.empty(max(need.value, 1), dtype=torch.uint8, device=cuda) if workspace else None
    out = torch.full((batch, hq, hd), 7.0, dtype=c["q"].dtype, device=cuda)
    _lib.check(L.bm_decode_attention(
        out.data_ptr(), d["q"].data_ptr(), d["kc"].data_ptr(), d["vc"].data_ptr(), d["seq_ids"].data_ptr(),
        d["lens"].data_ptr(), max_len, batch, hq, hkv, hd, max_seq, num_seqs, 0.0,
        None if ws is None else ws.data_ptr(), need.value if ws is not None else 0, ops.bm_dtype(c["q"]), status.ptr,
        torch.cuda.current_stream(cuda).cuda_stream))
    return out, d["kc"], d["vc"]


SHAPES = [
    (1, 6, 6, 48, 256, 1),         # the engine's decode step (tinyllama-shaped, heads = kv heads)
    (8, 32, 8, 64, 1024, 8),       # GQA group 4, several splits per sequence
    (3, 32, 2, 96, 700, 5),        # group 16, head_dim 96 (strided lanes), ragged max_seq
    (4, 64, 8, 128, 2048, 4),      # head_dim 128: the tensor-core / TMA kernels, two calls
]


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"b{s[0]}_h{s[1]}_{s[2]}_d{s[3]}" for s in SHAPES])
@pytest.mark.parametrize("pos_mode", ["last", "inside"])
def test_equals_the_two_calls_and_matches_the_oracle(cuda, dt, shape, pos_mode):
    batch, hq, hkv, hd, max_seq, num_seqs = shape
    c = case(cuda, dt, *shape, seed=batch * 100 + hd + (pos_mode == "inside"), pos_mode=pos_mode)
    table = ops.RopeTable(max_seq, hd, THETA, cuda)
    max_len = int(c["lens"].max())
    s1, s2 = ops.DeviceStatus(cuda), ops.DeviceStatus(cuda)
    got, kc1, vc1 = call_fused(cuda, c, table, max_len, s1)
    ref, kc2, vc2 = call_unfused(cuda, c, table, max_len, s2)
    torch.cuda.synchronize(cuda)
    assert s1.read() == 0 and s2.read() == 0
    assert bits_equal(kc1, kc2) and bits_equal(vc1, vc2)  # the same rows written, with the same bits
    assert bits_equal(got, ref)
    # the oracle: its RoPE + store, then its attention
    q2, kc_o, vc_o, bad = orc.rope_kv_store(to_np(c["q"]), to_np(c["k"]), to_np(c["v"]), c["positions"].numpy(),
                                            to_np(c["kc"]), to_np(c["vc"]), THETA, seq_ids=c["seq_ids"].numpy())
    assert bad == 0
    want, bad = oracle_attention(from_np(q2), from_np(kc_o), from_np(vc_o), c["seq_ids"], c["lens"])
    assert bad == 0
    assert orc.worst_error(to_np(got), want) <= TOL[dt]


def test_unsplit_without_workspace(cuda):
    c = case(cuda, torch.float32, 8, 32, 8, 64, 1024, 8, seed=5)
    table = ops.RopeTable(1024, 64, THETA, cuda)
    s1, s2 = ops.DeviceStatus(cuda), ops.DeviceStatus(cuda)
    got, kc1, _ = call_fused(cuda, c, table, 1024, s1, workspace=False)
    ref, kc2, _ = call_unfused(cuda, c, table, 1024, s2, workspace=False)
    torch.cuda.synchronize(cuda)
    assert s1.read() == 0 and bits_equal(got, ref) and bits_equal(kc1, kc2)


def test_a_bad_position_is_flagged_and_leaves_the_cache(cuda):
    """On the one-launch path a position at or past the query's length (the token
    would not be attended) is flagged; that token is neither rotated nor stored and
    its query attends over the cache as it is."""
    c = case(cuda, torch.float32, 4, 8, 4, 64, 512, 4, seed=9)
    c["positions"][1] = int(c["lens"][1])        # == len: not attended, so not the query's new token
    table = ops.RopeTable(512, 64, THETA, cuda)
    s = ops.DeviceStatus(cuda)
    got, kc1, vc1 = call_fused(cuda, c, table, 512, s)
    torch.cuda.synchronize(cuda)
    assert s.read() == _lib.BM_DEVERR_BAD_POSITION
    seq1 = int(c["seq_ids"][1])
    assert bits_equal(kc1[seq1], c["kc"][seq1].to(cuda)) and bits_equal(vc1[seq1], c["vc"][seq1].to(cuda))
    # query 1 with the unrotated q over the untouched cache; the others as usual
    want, _ = oracle_attention(c["q"][1:2], c["kc"], c["vc"], c["seq_ids"][1:2], c["lens"][1:2])
    assert orc.worst_error(to_np(got[1:2]), want) <= 1e-5

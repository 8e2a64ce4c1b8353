"""Decode attention (bm_decode_attention) against the oracle on the GPU.

The oracle restates the reference's attention check loop (tests/kernel_tests.cu:
229-258) in double precision, extended to GQA, batches and per-query lengths.
fp32 within 1e-5 and bf16 within 1e-2 in the reference's metric.
"""
import ctypes

import numpy as np
import pytest
import torch

from baremetalinferenceengine_b200 import _lib, ops
from oracle import oracle as orc
from tests.helpers import TOL, bits_equal, gen, randn, to_np

pytestmark = pytest.mark.gpu


def oracle_attention(q, kc, vc, seq_ids, lens):
    batch, hq, hd = q.shape
    num_seqs, hkv, max_seq, _ = kc.shape
    # every array the C call reads is bound to a name: a temporary's memory could be
    # freed before the call runs
    qn, kn, vn = to_np(q), to_np(kc), to_np(vc)
    sn = None if seq_ids is None else np.ascontiguousarray(seq_ids.numpy(), dtype=np.int32)
    ln = np.ascontiguousarray(lens.numpy(), dtype=np.int32)
    out = np.zeros_like(qn)
    bad = orc.lib().oracle_decode_attention(
        out.ctypes.data, qn.ctypes.data, kn.ctypes.data, vn.ctypes.data, None if sn is None else sn.ctypes.data,
        ln.ctypes.data, batch, hq, hkv, hd, max_seq, num_seqs, 0 if q.dtype == torch.float32 else 1)
    return out, bad


def run(cuda, q, kc, vc, seq_ids, lens, workspace=True, status=None, max_len=None):
    batch, hq, hd = q.shape
    num_seqs, hkv, max_seq, _ = kc.shape
    L = _lib.load()
    if max_len is None:
        max_len = int(lens.max()) if lens.numel() else 1
    need = ctypes.c_size_t()
    _lib.check(L.bm_decode_attention_workspace_size(batch, hq, hkv, hd, max_len, ctypes.byref(need)))
    ws = torch.empty(max(need.value, 1), dtype=torch.uint8, device=cuda) if workspace else None
    out = torch.full((batch, hq, hd), 7.0, dtype=q.dtype, device=cuda)
    qd, kd, vd = q.to(cuda), kc.to(cuda), vc.to(cuda)
    sd = None if seq_ids is None else seq_ids.to(cuda)
    ld = lens.to(cuda)
    _lib.check(L.bm_decode_attention(out.data_ptr(), qd.data_ptr(), kd.data_ptr(), vd.data_ptr(),
                                     None if sd is None else sd.data_ptr(), ld.data_ptr(), max_len, batch, hq, hkv,
                                     hd, max_seq, num_seqs, 0.0, None if ws is None else ws.data_ptr(),
                                     need.value if ws is not None else 0, ops.bm_dtype(q),
                                     None if status is None else status.ptr,
                                     torch.cuda.current_stream(cuda).cuda_stream))
    return out, need.value


ORACLE_DT = [torch.float32, torch.bfloat16]


@pytest.mark.parametrize("dt", ORACLE_DT, ids=["f32", "bf16"])
@pytest.mark.parametrize("batch,hq,hkv,hd,max_seq,num_seqs", [
    (1, 6, 6, 48, 256, 1),        # tinyllama: the reference's own shape (heads = kv heads)
    (16, 32, 8, 128, 8192, 16),   # Llama-3-8B decode, GQA group 4
    (4, 64, 8, 128, 8192, 4),     # Llama-3-70B decode, GQA group 8
    (3, 32, 2, 64, 1024, 5),      # group 16, head_dim 64
    (2, 4, 4, 256, 600, 2),       # head_dim 256
])
@pytest.mark.parametrize("workspace", [True, False], ids=["split", "unsplit"])
def test_decode_attention_matches_oracle(cuda, dt, batch, hq, hkv, hd, max_seq, num_seqs, workspace):
    g = gen(batch * 1000 + hq + hd)
    q = randn((batch, hq, hd), dt, g)
    kc = randn((num_seqs, hkv, max_seq, hd), dt, g)
    vc = randn((num_seqs, hkv, max_seq, hd), dt, g)
    seq_ids = torch.randint(0, num_seqs, (batch,), generator=g, dtype=torch.int32)
    lens = torch.randint(1, max_seq + 1, (batch,), generator=g, dtype=torch.int32)
    lens[0] = max_seq  # the full cache
    if batch > 1:
        lens[1] = 1  # a single position
    out, need = run(cuda, q, kc, vc, seq_ids, lens, workspace)
    want, bad = oracle_attention(q, kc, vc, seq_ids, lens)
    assert bad == 0
    assert orc.worst_error(to_np(out), want) <= TOL[dt]


@pytest.mark.parametrize("dt", ORACLE_DT, ids=["f32", "bf16"])
@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 8), (32, 8), (64, 8), (32, 2)],
                         ids=["group1", "group2", "group4", "group8", "group16"])
@pytest.mark.parametrize("workspace", [True, False], ids=["split", "unsplit"])
def test_head_dim_128_tile_edges_and_stale_cache(cuda, dt, hq, hkv, workspace):
    """head_dim 128 (bf16: the tensor-core kernel, 128-position tiles; fp32: the
    TMA-fed kernel, 64-position tiles): lengths at and around the tile edges,
    every GQA group size, and cache slots past each length holding NaN, which
    must not reach the output."""
    batch, hd, max_seq = 12, 128, 1024
    g = gen(hq * 31 + hkv + (7 if workspace else 0))
    q = randn((batch, hq, hd), dt, g)
    kc = randn((batch, hkv, max_seq, hd), dt, g)
    vc = randn((batch, hkv, max_seq, hd), dt, g)
    lens = torch.tensor([1, 63, 64, 65, 127, 128, 129, 255, 256, 257, 1000, 1024], dtype=torch.int32)
    for b in range(batch):  # stale slots: NaN past the length
        kc[b, :, int(lens[b]):, :] = float("nan")
        vc[b, :, int(lens[b]):, :] = float("nan")
    seq_ids = torch.arange(batch, dtype=torch.int32)
    out, _ = run(cuda, q, kc, vc, seq_ids, lens, workspace)
    want, bad = oracle_attention(q, kc, vc, seq_ids, lens)
    assert bad == 0
    assert torch.isfinite(out.float()).all()
    assert orc.worst_error(to_np(out), want) <= TOL[dt]


@pytest.mark.parametrize("max_seq,lens", [
    (8192, [8192]),             # one 8192-position sequence: 16 splits per (query, kv head)
    (8192, [8192, 300]),        # a second, short query: its splits past 300 positions are empty
    (1024, [1024, 1, 700]),     # 2 splits per query
    (32768, [32768, 20000]),    # 64 splits per (query, kv head)
])
@pytest.mark.parametrize("workspace", [True, False], ids=["ws", "no_ws"])
def test_tensor_core_few_pairs_long_sequences(cuda, max_seq, lens, workspace):
    """bf16 head_dim 128 with fewer (query, kv head) pairs than the balanced kernel
    takes: the per-pair grid splits each sequence (up to 64 splits, merged through
    the workspace) or, without a workspace, runs each pair whole. Stale NaN past
    each length stays out."""
    batch, hq, hkv, hd = len(lens), 32, 8, 128
    g = gen(max_seq + batch)
    q = randn((batch, hq, hd), torch.bfloat16, g)
    kc = randn((batch, hkv, max_seq, hd), torch.bfloat16, g)
    vc = randn((batch, hkv, max_seq, hd), torch.bfloat16, g)
    lens = torch.tensor(lens, dtype=torch.int32)
    for b in range(batch):
        kc[b, :, int(lens[b]):, :] = float("nan")
        vc[b, :, int(lens[b]):, :] = float("nan")
    seq_ids = torch.arange(batch, dtype=torch.int32)
    status = ops.DeviceStatus(cuda)
    out, _ = run(cuda, q, kc, vc, seq_ids, lens, workspace, status=status)
    assert status.read() == 0
    want, bad = oracle_attention(q, kc, vc, seq_ids, lens)
    assert bad == 0
    assert torch.isfinite(out.float()).all()
    assert orc.worst_error(to_np(out), want) <= TOL[torch.bfloat16]


@pytest.mark.parametrize("dt", ORACLE_DT, ids=["f32", "bf16"])
def test_stale_workspace_contents_do_not_leak(cuda, dt):
    """Splits that lie past a query's length write only their (max, sum); the
    output slots of such a split keep whatever the workspace held. Filled with
    NaN bytes first, the workspace must still give the oracle's results."""
    batch, hq, hkv, hd, max_seq = 6, 32, 8, 128, 8192
    g = gen(77)
    q = randn((batch, hq, hd), dt, g)
    kc = randn((batch, hkv, max_seq, hd), dt, g)
    vc = randn((batch, hkv, max_seq, hd), dt, g)
    lens = torch.tensor([max_seq, 1, 100, 513, 2000, 7000], dtype=torch.int32)  # most splits of short queries empty
    seq_ids = torch.arange(batch, dtype=torch.int32)
    L = _lib.load()
    need = ctypes.c_size_t()
    _lib.check(L.bm_decode_attention_workspace_size(batch, hq, hkv, hd, max_seq, ctypes.byref(need)))
    assert need.value > 0
    ws = torch.full((need.value,), 0xFF, dtype=torch.uint8, device=cuda)  # every float a NaN
    out = torch.empty((batch, hq, hd), dtype=dt, device=cuda)
    qd, kd, vd, sd, ld = q.to(cuda), kc.to(cuda), vc.to(cuda), seq_ids.to(cuda), lens.to(cuda)
    _lib.check(L.bm_decode_attention(out.data_ptr(), qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), sd.data_ptr(),
                                     ld.data_ptr(), max_seq, batch, hq, hkv, hd, max_seq, batch, 0.0, ws.data_ptr(),
                                     need.value, ops.bm_dtype(q), None, torch.cuda.current_stream(cuda).cuda_stream))
    torch.cuda.synchronize(cuda)
    assert torch.isfinite(out.float()).all()
    want, bad = oracle_attention(q, kc, vc, seq_ids, lens)
    assert bad == 0
    assert orc.worst_error(to_np(out), want) <= TOL[dt]


def test_reference_attention_cases(cuda):
    """The reference's three attention checks (tests/kernel_tests.cu:285-287):
    inputs U[-1,1], one query, heads = kv heads."""
    for heads, hd, max_seq, seq_len in [(1, 16, 1, 1), (6, 48, 256, 1), (6, 48, 256, 200)]:
        g = gen(heads + seq_len)
        q = torch.rand(1, heads, hd, generator=g) * 2 - 1
        kc = torch.rand(1, heads, max_seq, hd, generator=g) * 2 - 1
        vc = torch.rand(1, heads, max_seq, hd, generator=g) * 2 - 1
        lens = torch.tensor([seq_len], dtype=torch.int32)
        out, _ = run(cuda, q, kc, vc, None, lens)
        want, _ = oracle_attention(q, kc, vc, None, lens)
        assert orc.worst_error(to_np(out), want) <= 1e-5


def test_bad_entries_are_skipped_and_flagged(cuda):
    g = gen(9)
    q = torch.randn(4, 8, 64, generator=g)
    kc, vc = torch.randn(2, 2, 32, 64, generator=g), torch.randn(2, 2, 32, 64, generator=g)
    seq_ids = torch.tensor([0, 2, 1, -1], dtype=torch.int32)
    lens = torch.tensor([5, 5, 0, 3], dtype=torch.int32)
    status = ops.DeviceStatus(cuda)
    out, _ = run(cuda, q, kc, vc, seq_ids, lens, status=status)
    assert status.read() == _lib.BM_DEVERR_BAD_SEQUENCE | _lib.BM_DEVERR_BAD_POSITION
    want, bad = oracle_attention(q, kc, vc, seq_ids, lens)
    assert bad == _lib.BM_DEVERR_BAD_SEQUENCE | _lib.BM_DEVERR_BAD_POSITION
    outc = out.cpu()
    assert orc.worst_error(outc[0].numpy(), want[0]) <= 1e-5
    for b in (1, 2, 3):
        assert bits_equal(outc[b], torch.full((8, 64), 7.0))


@pytest.mark.parametrize("path,dt,batch,hq,hkv,hd", [
    ("cuda_cores_f32", torch.float32, 4, 8, 2, 64),
    ("cuda_cores_bf16", torch.bfloat16, 4, 8, 2, 64),
    ("tensor_cores_per_pair_grid", torch.bfloat16, 4, 8, 2, 128),  # 8 pairs: below the balanced minimum
    ("tensor_cores_balanced", torch.bfloat16, 8, 8, 8, 128),  # 64 pairs, with a workspace
    ("f32_tma", torch.float32, 4, 8, 2, 128),
])
def test_lengths_beyond_max_len_are_flagged_on_every_path(cuda, path, dt, batch, hq, hkv, hd):
    """max_len bounds every query's length: the split plans cover max_len
    positions, so a longer query (still within max_seq) is flagged
    BM_DEVERR_BAD_POSITION and skipped on every path, never cut short."""
    g = gen(hd + batch)
    max_seq, max_len = 2048, 1000
    q = randn((batch, hq, hd), dt, g)
    kc, vc = randn((batch, hkv, max_seq, hd), dt, g), randn((batch, hkv, max_seq, hd), dt, g)
    lens = torch.tensor(([2048, 600, 1000, 1001, 300, 999, 1500, 1][:batch]), dtype=torch.int32)
    seq_ids = torch.arange(batch, dtype=torch.int32)
    status = ops.DeviceStatus(cuda)
    out, _ = run(cuda, q, kc, vc, seq_ids, lens, status=status, max_len=max_len)
    assert status.read() == _lib.BM_DEVERR_BAD_POSITION
    ok = lens <= max_len
    want, _ = oracle_attention(q[ok], kc, vc, seq_ids[ok], lens[ok])
    outc = out.cpu()
    assert orc.worst_error(to_np(outc[ok]), want) <= TOL[dt]
    for b in torch.nonzero(~ok).flatten().tolist():
        assert bits_equal(outc[b], torch.full((hq, hd), 7.0, dtype=dt)), b


def test_workspace_size_and_argument_checks(cuda):
    L = _lib.load()
    n = ctypes.c_size_t()
    _lib.check(L.bm_decode_attention_workspace_size(1, 8, 8, 128, 8192, ctypes.byref(n)))
    assert n.value > 0  # one long query is split across CTAs
    _lib.check(L.bm_decode_attention_workspace_size(1, 8, 8, 128, 100, ctypes.byref(n)))
    assert n.value == 0  # a single tile needs no split
    dummy = torch.zeros(64, device=cuda)
    p = dummy.data_ptr()
    lens = torch.ones(1, dtype=torch.int32, device=cuda)
    for args in [(1, 6, 4, 64), (1, 32, 1, 64), (1, 8, 8, 300), (1, 8, 8, 34)]:
        st = L.bm_decode_attention(p, p, p, p, None, lens.data_ptr(), 1, args[0], args[1], args[2], args[3], 8, 1,
                                   0.0, None, 0, 0, None, None)
        assert st == _lib.BM_ERR_INVALID_ARGUMENT, args


@pytest.mark.parametrize("batch,hq,hkv,max_seq,lens", [
    (1, 32, 8, 8192, [8192]),            # one 8192-position sequence: 8 pairs, 16 splits each
    (2, 64, 8, 8192, [5000, 8192]),      # two ragged 70B queries
    (3, 32, 8, 4096, [4096, 700, 1]),    # a query whose splits are mostly empty
])
def test_tensor_core_grid_with_a_stale_workspace(cuda, batch, hq, hkv, max_seq, lens):
    """Below the balanced kernel's minimum, bf16 head_dim 128 runs the per-(query,
    kv head, split) tensor-core grid, its splits' partials passing through the
    caller's workspace to the merge kernel. A workspace holding garbage, a zeroed
    one, and the previous call's leftovers give the same bits, within the tolerance
    of the oracle: no path reads a slot that the call did not write first."""
    dt, hd = torch.bfloat16, 128
    g = gen(batch * 31 + hq)
    q = randn((batch, hq, hd), dt, g)
    kc, vc = randn((batch, hkv, max_seq, hd), dt, g), randn((batch, hkv, max_seq, hd), dt, g)
    seq_ids = torch.arange(batch, dtype=torch.int32)
    lens_t = torch.tensor(lens, dtype=torch.int32)
    L = _lib.load()
    need = ctypes.c_size_t()
    _lib.check(L.bm_decode_attention_workspace_size(batch, hq, hkv, hd, max_seq, ctypes.byref(need)))
    ws = torch.empty(need.value, dtype=torch.uint8, device=cuda)
    qd, kd, vd, sd, ld = q.to(cuda), kc.to(cuda), vc.to(cuda), seq_ids.to(cuda), lens_t.to(cuda)
    status = ops.DeviceStatus(cuda)
    outs = []
    for fill in (0xFF, 0x00, None):  # garbage, zeros, and the previous call's leftovers
        if fill is not None:
            ws.fill_(fill)
        out = torch.full((batch, hq, hd), 7.0, dtype=dt, device=cuda)
        _lib.check(L.bm_decode_attention(out.data_ptr(), qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), sd.data_ptr(),
                                         ld.data_ptr(), max_seq, batch, hq, hkv, hd, max_seq, batch, 0.0,
                                         ws.data_ptr(), need.value, ops.bm_dtype(q), status.ptr,
                                         torch.cuda.current_stream(cuda).cuda_stream))
        outs.append(out.cpu())
    torch.cuda.synchronize(cuda)
    assert status.read() == 0
    assert bits_equal(outs[0], outs[1]) and bits_equal(outs[1], outs[2])
    want, bad = oracle_attention(q, kc, vc, seq_ids, lens_t)
    assert bad == 0
    assert orc.worst_error(to_np(outs[2]), want) <= TOL[dt]

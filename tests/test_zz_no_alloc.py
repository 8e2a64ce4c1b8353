"""The allocation-free decode attention (bm_decode_attention_static_scratch).

This entry point exists for callers that cannot call cudaMalloc (for example an
application whose own arena owns all device memory, or a plugin in a process that
reserved the GPU up front): it keeps the split partials in a fixed 8 MiB array
inside the library instead of a caller-allocated workspace. These tests call it
through the C ABI on two calls in a row (the array keeps the first call's
contents) and check each call's output against the oracle (the reference's
attention check loop, tests/kernel_tests.cu:229-258, restated in double
precision for batches and GQA) within the suite's tolerance, and bit for bit
against bm_decode_attention given a workspace of the array's size (the same
plan). They also check that the arguments are validated first, that the size
limit follows the plan actually run, and that a batch needing more scratch
than the array holds is refused. The file is named to be collected last.
"""
import ctypes

import pytest
import torch

from baremetalinferenceengine_b200 import _lib, ops
from oracle import oracle as orc
from tests.helpers import TOL, bits_equal, gen, randn, to_np
from tests.test_gpu_attention import oracle_attention

pytestmark = pytest.mark.gpu

STATIC_SCRATCH_BYTES = 8 << 20


def _case(dt, seed, batch, hq, hkv, hd=128, max_seq=8192):
    g = gen(seed)
    q = randn((batch, hq, hd), dt, g)
    kc = randn((batch, hkv, max_seq, hd), dt, g)
    vc = randn((batch, hkv, max_seq, hd), dt, g)
    seq_ids = torch.arange(batch, dtype=torch.int32)
    lens = torch.randint(1, max_seq + 1, (batch,), generator=g, dtype=torch.int32)
    lens[0] = max_seq
    return q, kc, vc, seq_ids, lens


def _with_workspace(L, cuda, dev, max_len, ws_bytes):
    q, kc, vc, seq_ids, lens = dev
    batch, hq, hd = q.shape
    _, hkv, max_seq, _ = kc.shape
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
    out = torch.full_like(q, float("nan"))
    _lib.check(L.bm_decode_attention(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), seq_ids.data_ptr(),
                                     lens.data_ptr(), max_len, batch, hq, hkv, hd, max_seq, kc.shape[0], 0.0,
                                     ws.data_ptr(), ws_bytes, ops.bm_dtype(q), None,
                                     torch.cuda.current_stream(cuda).cuda_stream))
    return out


def _static(L, cuda, dev, max_len, status=None):
    q, kc, vc, seq_ids, lens = dev
    batch, hq, hd = q.shape
    _, hkv, max_seq, _ = kc.shape
    out = torch.full_like(q, float("nan"))
    st = L.bm_decode_attention_static_scratch(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                              seq_ids.data_ptr(), lens.data_ptr(), max_len, batch, hq, hkv, hd,
                                              max_seq, kc.shape[0], 0.0, ops.bm_dtype(q),
                                              None if status is None else status.ptr,
                                              torch.cuda.current_stream(cuda).cuda_stream)
    return st, out


@pytest.mark.parametrize("dt,batch,hq,hkv", [
    (torch.bfloat16, 4, 32, 8),  # 32 (query, kv head) pairs: the balanced tensor-core kernel
    (torch.bfloat16, 2, 32, 8),  # 16 pairs: the per-pair tensor-core grid, split sequences
    (torch.float32, 4, 32, 8),   # fp32: the TMA-fed CUDA-core grid, split sequences
], ids=["bf16-balanced", "bf16-grid", "f32-grid"])
def test_two_calls_in_a_row_match_the_oracle(cuda, dt, batch, hq, hkv):
    L = _lib.load()
    for call, seed in enumerate((101, 202)):  # different inputs each time: stale scratch must not leak
        host = _case(dt, seed, batch, hq, hkv)
        max_len = int(host[4].max())
        need = ctypes.c_size_t()
        _lib.check(L.bm_decode_attention_workspace_size(batch, hq, hkv, 128, max_len, ctypes.byref(need)))
        assert 0 < need.value <= STATIC_SCRATCH_BYTES  # this batch uses scratch, so the static array is used
        dev = tuple(t.to(cuda) for t in host)
        status = ops.DeviceStatus(cuda)
        st, got = _static(L, cuda, dev, max_len, status)
        assert st == _lib.BM_OK, L.bm_last_error_message()
        assert status.read() == 0
        want, bad = oracle_attention(*host)
        assert bad == 0
        assert orc.worst_error(to_np(got), want) <= TOL[dt], f"call {call}"
        # the workspace entry point given as much scratch runs the same plan: the same bits
        same_plan = _with_workspace(L, cuda, dev, max_len, STATIC_SCRATCH_BYTES)
        torch.cuda.synchronize(cuda)
        assert bits_equal(got, same_plan), f"call {call}"


def test_the_limit_follows_the_plan_that_runs(cuda):
    """fp32 head_dim 128 keeps at least four 128-position tiles per split, so 512
    positions run unsplit and need no scratch, even though the conservative
    bm_decode_attention_workspace_size figure for this batch (8.5 MB) is above the
    array's 8 MiB."""
    L = _lib.load()
    batch, hq, hkv, max_seq = 64, 128, 8, 512
    need = ctypes.c_size_t()
    _lib.check(L.bm_decode_attention_workspace_size(batch, hq, hkv, 128, max_seq, ctypes.byref(need)))
    assert need.value > STATIC_SCRATCH_BYTES
    host = _case(torch.float32, 7, batch, hq, hkv, max_seq=max_seq)
    dev = tuple(t.to(cuda) for t in host)
    st, got = _static(L, cuda, dev, int(host[4].max()))
    assert st == _lib.BM_OK, L.bm_last_error_message()
    torch.cuda.synchronize(cuda)
    want, _ = oracle_attention(*host)
    assert orc.worst_error(to_np(got), want) <= TOL[torch.float32]


def test_arguments_are_checked_before_the_size(cuda):
    L = _lib.load()
    dummy = torch.zeros(16, device=cuda)
    p = dummy.data_ptr()
    lens = torch.ones(1, dtype=torch.int32, device=cuda)
    for batch, hq, hkv, hd in [(70000, 8, 8, 128), (1, 6, 4, 128), (1, 8, 8, 300)]:
        st = L.bm_decode_attention_static_scratch(p, p, p, p, None, lens.data_ptr(), 8192, batch, hq, hkv, hd, 8192,
                                                  1, 0.0, 0, None, None)
        assert st == _lib.BM_ERR_INVALID_ARGUMENT
        assert b"static array" not in L.bm_last_error_message(), (batch, hq, hkv, hd)


def test_a_batch_needing_more_scratch_is_refused(cuda):
    L = _lib.load()
    batch, hq, hkv, hd, max_len = 8, 128, 8, 256, 8192
    dummy = torch.zeros(16, device=cuda)
    p = dummy.data_ptr()
    lens = torch.full((batch,), max_len, dtype=torch.int32, device=cuda)
    st = L.bm_decode_attention_static_scratch(p, p, p, p, None, lens.data_ptr(), max_len, batch, hq, hkv, hd,
                                              max_len, 1, 0.0, 0, None, None)
    assert st == _lib.BM_ERR_INVALID_ARGUMENT
    assert b"static array" in L.bm_last_error_message()

"""The allocation-free decode attention (bm_decode_attention_static_scratch).

This entry point exists for callers that cannot call cudaMalloc (for example an
application whose own arena owns all device memory, or a plugin in a process that
reserved the GPU up front): it keeps the split partials in a fixed 8 MiB array
inside the library instead of a caller-allocated workspace. These tests call it
through the C ABI and compare it with bm_decode_attention given a workspace, on
two calls in a row (the array keeps the first call's contents), and check that a
batch needing more scratch than the array holds is refused. The file is named to
be collected last.
"""
import ctypes

import pytest
import torch

from baremetalinferenceengine_b200 import _lib, ops
from oracle import oracle as orc
from tests.helpers import TOL, gen, randn, to_np

pytestmark = pytest.mark.gpu

STATIC_SCRATCH_BYTES = 8 << 20


def _case(cuda, dt, seed, batch=4, hq=32, hkv=8, hd=128, max_seq=8192):
    g = gen(seed)
    q = randn((batch, hq, hd), dt, g).to(cuda)
    kc = randn((batch, hkv, max_seq, hd), dt, g).to(cuda)
    vc = randn((batch, hkv, max_seq, hd), dt, g).to(cuda)
    seq_ids = torch.arange(batch, dtype=torch.int32, device=cuda)
    lens = torch.randint(1, max_seq + 1, (batch,), generator=g, dtype=torch.int32)
    lens[0] = max_seq
    return q, kc, vc, seq_ids, lens.to(cuda), int(lens.max())


def _with_workspace(L, cuda, q, kc, vc, seq_ids, lens, max_len):
    batch, hq, hd = q.shape
    _, hkv, max_seq, _ = kc.shape
    need = ctypes.c_size_t()
    _lib.check(L.bm_decode_attention_workspace_size(batch, hq, hkv, hd, max_len, ctypes.byref(need)))
    ws = torch.empty(max(need.value, 1), dtype=torch.uint8, device=cuda)
    out = torch.empty_like(q)
    _lib.check(L.bm_decode_attention(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), seq_ids.data_ptr(),
                                     lens.data_ptr(), max_len, batch, hq, hkv, hd, max_seq, kc.shape[0], 0.0,
                                     ws.data_ptr(), need.value, ops.bm_dtype(q), None,
                                     torch.cuda.current_stream(cuda).cuda_stream))
    return out, need.value


def _static(L, cuda, q, kc, vc, seq_ids, lens, max_len):
    batch, hq, hd = q.shape
    _, hkv, max_seq, _ = kc.shape
    out = torch.full_like(q, float("nan"))
    st = L.bm_decode_attention_static_scratch(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                              seq_ids.data_ptr(), lens.data_ptr(), max_len, batch, hq, hkv, hd,
                                              max_seq, kc.shape[0], 0.0, ops.bm_dtype(q), None,
                                              torch.cuda.current_stream(cuda).cuda_stream)
    return st, out


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
def test_two_calls_in_a_row_match_the_workspace_entry_point(cuda, dt):
    L = _lib.load()
    for call, seed in enumerate((101, 202)):  # different inputs each time: stale scratch must not leak
        q, kc, vc, seq_ids, lens, max_len = _case(cuda, dt, seed)
        want, need = _with_workspace(L, cuda, q, kc, vc, seq_ids, lens, max_len)
        assert 0 < need <= STATIC_SCRATCH_BYTES  # this batch is split, so the static array is used
        st, got = _static(L, cuda, q, kc, vc, seq_ids, lens, max_len)
        assert st == _lib.BM_OK, L.bm_last_error_message()
        torch.cuda.synchronize(cuda)
        assert orc.worst_error(to_np(got), to_np(want)) <= TOL[dt], f"call {call}"


def test_a_batch_needing_more_scratch_is_refused(cuda):
    L = _lib.load()
    batch, hq, hkv, hd, max_len = 8, 128, 8, 256, 8192
    need = ctypes.c_size_t()
    _lib.check(L.bm_decode_attention_workspace_size(batch, hq, hkv, hd, max_len, ctypes.byref(need)))
    assert need.value > STATIC_SCRATCH_BYTES
    dummy = torch.zeros(16, device=cuda)
    p = dummy.data_ptr()
    lens = torch.full((batch,), max_len, dtype=torch.int32, device=cuda)
    st = L.bm_decode_attention_static_scratch(p, p, p, p, None, lens.data_ptr(), max_len, batch, hq, hkv, hd,
                                              max_len, 1, 0.0, 0, None, None)
    assert st == _lib.BM_ERR_INVALID_ARGUMENT
    assert b"static array" in L.bm_last_error_message()

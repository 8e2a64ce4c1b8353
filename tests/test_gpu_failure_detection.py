"""Failure detection on the GPU without a GPU fault.

Every tensor-core kernel bounds its mbarrier waits in time (and in polls): a wait
that runs out ORs BM_DEVERR_TIMEOUT into the caller's status word and the kernel
finishes instead of hanging. bm_selftest_bounded_wait makes one such wait run
out on purpose - a barrier that nothing ever completes, with a short limit - and
these tests check the status the host reads, the time the wait took, that a
second waiter honouring the abort gives up at once, and that the context is
still usable afterwards.
"""
import pytest
import torch

from baremetalinferenceengine_b200 import _lib, ops
from oracle import oracle as orc
from tests.helpers import gen, randn, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("limit_ms", [20, 200])
def test_a_wait_that_runs_out_reports_timeout_and_the_context_survives(cuda, limit_ms):
    L = _lib.load()
    status = ops.DeviceStatus(cuda)
    result = torch.full((4,), -1, dtype=torch.int64, device=cuda)
    limit_ns = limit_ms * 1_000_000
    _lib.check(L.bm_selftest_bounded_wait(limit_ns, status.ptr, result.data_ptr(),
                                          torch.cuda.current_stream(cuda).cuda_stream))
    torch.cuda.synchronize(cuda)
    assert status.read() == _lib.BM_DEVERR_TIMEOUT
    ok1, took1, ok2, took2 = result.cpu().tolist()
    assert ok1 == 0 and ok2 == 0
    assert limit_ns <= took1 < limit_ns + 500_000_000  # gave up at the limit, not before, not much after
    assert took2 < 5_000_000  # the abort flag was honoured at once

    # the context still runs kernels: a SwiGLU against the oracle
    g = gen(limit_ms)
    gate, up = randn((4, 256), torch.float32, g), randn((4, 256), torch.float32, g)
    out = ops.swiglu(gate.to(cuda), up.to(cuda))
    torch.cuda.synchronize(cuda)
    assert orc.worst_error(to_np(out), orc.swiglu(to_np(gate), to_np(up))) <= 1e-5

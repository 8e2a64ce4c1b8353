"""bm_rmsnorm_gemm: the RMSNorm before a projection and the projection together.

The oracle composes the reference's own steps: the residual add and RMSNorm of its
check loops (tests/kernel_tests.cu:75-79, 206; the engine's order at
src/execution_engine.cu:118-121) and its GEMM (reference_gemm, tests/kernel_tests.cu:
49-59), then the SwiGLU (:122). fp32 within 1e-5 in the reference's metric
|got - want| / (1 + |want|), the updated residual bit-exact (one fp32 add), and the
same within 1e-5 of the unfused calls (bm_add_rmsnorm, then bm_gemm_shared_a or
bm_gemm_swiglu): the fused form sums the squares in another order, so the norm can
differ in the last bit.
"""
import numpy as np
import pytest
import torch

from baremetalinferenceengine_b200 import _lib, ops
from oracle import oracle as orc
from tests.helpers import gen, to_np

pytestmark = pytest.mark.gpu

EPS = 1e-5


def inputs(m, k, widths, seed, with_d=True):
    g = gen(seed)
    h = torch.randn(m, k, generator=g)
    d = torch.randn(m, k, generator=g) if with_d else None
    w = 1 + 0.02 * torch.randn(k, generator=g)
    bs = [(torch.rand(k, n, generator=g) * 2 - 1) * (2.0 / k ** 0.5) for n in widths]
    return h, d, w, bs


def oracle_products(h, d, w, bs, swiglu):
    if d is not None:
        x, y = orc.add_rmsnorm(h.numpy(), d.numpy(), w.numpy(), EPS)
    else:
        x, y = h.numpy(), orc.rmsnorm(h.numpy(), w.numpy(), EPS)
    y = np.asarray(y, dtype=np.float32)
    if swiglu:
        return x, [orc.gemm_swiglu(y, bs[0].numpy(), bs[1].numpy(), threads=8)]
    return x, [orc.gemm(y, b.numpy(), threads=8) for b in bs]


@pytest.mark.parametrize("m,k,widths,with_d,swiglu,keep_residual", [
    (1, 288, (288, 288, 288), True, False, True),    # the engine's Q, K, V after the residual add
    (1, 288, (288, 288, 288), False, False, False),  # layer 0: the norm of the embedding row alone
    (1, 288, (768, 768), True, True, True),          # the engine's gate and up with the SwiGLU
    (1, 288, (32000,), True, False, False),          # the final norm and the vocabulary product
    (3, 4096, (4096, 1024, 1024), True, False, True),  # Llama-3-8B Q, K, V, three tokens
    (9, 130, (201,), True, False, True),             # two row tiles, ragged widths (scalar B loads)
    (64, 512, (1000, 1000), True, True, True),       # the SwiGLU over 16 row tiles of 4
    (512, 4096, (640,), True, False, True),          # rows too long for shared memory: two launches
])
def test_matches_the_oracle_and_the_unfused_calls(cuda, m, k, widths, with_d, swiglu, keep_residual):
    h, d, w, bs = inputs(m, k, widths, seed=m * 31 + k + len(widths), with_d=with_d)
    hd, dd, wd, bsd = h.to(cuda), (d.to(cuda) if d is not None else None), w.to(cuda), [b.to(cuda) for b in bs]
    res = torch.full((m, k), float("nan"), device=cuda) if keep_residual and with_d else None
    outs = ops.rmsnorm_gemm(hd, wd, bsd, d=dd, eps=EPS, swiglu=swiglu, residual_out=res)
    # unfused: the residual add and norm, then the products
    h2 = hd.clone()
    normed = torch.empty_like(hd)
    if dd is not None:
        ops.add_rmsnorm(h2, dd, wd, EPS, out=normed)
    else:
        ops.rmsnorm(hd, wd, EPS, out=normed)
    unfused = [ops.gemm_swiglu(normed, bsd[0], bsd[1])] if swiglu else ops.gemm_shared_a(normed, bsd)
    torch.cuda.synchronize(cuda)
    x_want, want = oracle_products(h, d, w, bs, swiglu)
    assert len(outs) == len(want)
    for got, ref, plain in zip(outs, want, unfused):
        assert orc.worst_error(to_np(got), ref) <= 1e-5
        assert orc.worst_error(to_np(got), to_np(plain)) <= 1e-5
    if res is not None:
        assert np.array_equal(to_np(res), x_want)      # h + d, one fp32 add
    assert torch.equal(hd.cpu(), h)                    # h itself is never written
    out2 = ops.rmsnorm_gemm(hd, wd, bsd, d=dd, eps=EPS, swiglu=swiglu)
    torch.cuda.synchronize(cuda)
    for a, b in zip(outs, out2):                       # deterministic: fixed order everywhere
        assert torch.equal(a, b)


def test_bf16_runs_the_norm_then_the_tensor_core_products(cuda):
    m, k, widths = 4, 256, (256, 128)
    h, d, w, bs = inputs(m, k, widths, seed=7)
    dt = torch.bfloat16
    hd, dd, wd = h.to(cuda).to(dt), d.to(cuda).to(dt), w.to(cuda).to(dt)
    bsd = [b.to(cuda).to(dt) for b in bs]
    res = torch.empty(m, k, device=cuda, dtype=dt)
    outs = ops.rmsnorm_gemm(hd, wd, bsd, d=dd, eps=EPS, residual_out=res)
    torch.cuda.synchronize(cuda)
    x, y = orc.add_rmsnorm(to_np(hd), to_np(dd), to_np(wd), EPS)
    assert np.array_equal(to_np(res), x)
    for got, b in zip(outs, bsd):
        want = orc.gemm(y, to_np(b), threads=8)
        assert orc.worst_error(to_np(got), want) <= 1e-2


def test_a_residual_output_over_its_inputs_is_refused(cuda):
    m, k = 2, 64
    h, d, w, bs = inputs(m, k, (64,), seed=3)
    hd, dd, wd, bsd = h.to(cuda), d.to(cuda), w.to(cuda), [b.to(cuda) for b in bs]
    with pytest.raises(ops.BMError) as e:
        ops.rmsnorm_gemm(hd, wd, bsd, d=dd, residual_out=hd)
    assert e.value.status == _lib.BM_ERR_INVALID_ARGUMENT
    with pytest.raises(ops.BMError):
        ops.rmsnorm_gemm(hd, wd, bsd[:1] * 3, d=dd, swiglu=True)  # swiglu takes two weights

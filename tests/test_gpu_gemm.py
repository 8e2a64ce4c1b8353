"""Tensor-core GEMM and fused GEMM + SwiGLU (bm_gemm, bm_gemm_swiglu) on the GPU.

The oracle's GEMM restates the reference's reference_gemm (tests/kernel_tests.cu:
49-59) and is pinned to it bit for bit; tests/golden/gemm_reference.npz holds the
reference's own outputs on bf16-representable inputs. The kernels take bf16
operands, accumulate in fp32 and round the result once to bf16, so the bar is the
bf16 one: |got - want| / (1 + |want|) <= 1e-2.
"""
import numpy as np
import pytest
import torch

from baremetalinferenceengine_b200 import _lib, ops
from oracle import oracle as orc
from tests.helpers import bits_equal, from_np, gen, to_np

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2
GOLDEN = "tests/golden/gemm_reference.npz"


def _uniform(shape, lo, hi, g):
    return (torch.rand(shape, generator=g) * (hi - lo) + lo).to(torch.bfloat16)


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_gemm_matches_the_reference_outputs(cuda, golden):
    for n in range(int(golden["count"])):
        a = from_np(golden[f"a{n}"], cuda)
        b = from_np(golden[f"b{n}"], cuda)
        got = ops.gemm(a, b)
        torch.cuda.synchronize(cuda)
        err = orc.worst_error(to_np(got), golden[f"c{n}"])
        assert err <= BF16_TOL, (n, tuple(a.shape), tuple(b.shape), err)


def test_gemm_swiglu_matches_the_reference_products(cuda, golden):
    x, wg, wu = (from_np(golden[k], cuda) for k in ("ffn_x", "ffn_w_gate", "ffn_w_up"))
    got = ops.gemm_swiglu(x, wg, wu)
    torch.cuda.synchronize(cuda)
    want = orc.swiglu(golden["ffn_gate"], golden["ffn_up"])  # the reference's SwiGLU of its GEMM outputs
    assert orc.worst_error(to_np(got), want) <= BF16_TOL


@pytest.mark.parametrize("m,n,k", [
    (1, 4096, 4096),      # the reference's decode-shaped test_gemm (tests/kernel_tests.cu:267)
    (16, 16, 16),
    (128, 256, 64),       # exactly one tile and one K step
    (257, 264, 136),      # ragged in every dimension
    (300, 520, 1000),
    (64, 1024, 4096),     # decode batch: one row block, long K
    (1024, 768, 512),     # several row blocks per column block
])
def test_gemm_matches_the_oracle(cuda, m, n, k):
    g = gen(m * 7 + n * 3 + k)
    a = _uniform((m, k), -1.0, 1.0, g)
    b = _uniform((k, n), -1.0, 1.0, g)
    got = ops.gemm(a.to(cuda), b.to(cuda))
    torch.cuda.synchronize(cuda)
    want = orc.gemm(to_np(a), to_np(b).copy(), threads=8)
    assert orc.worst_error(to_np(got), want) <= BF16_TOL


@pytest.mark.parametrize("rows,dim,hidden", [
    (1, 4096, 1024),      # one decode token
    (64, 4096, 1024),     # a decode batch
    (200, 264, 136),      # ragged
    (129, 512, 384),      # one row past a row block
    (512, 2048, 2048),
    (8, 8, 8),            # the smallest legal shape
])
def test_gemm_swiglu_matches_the_oracle(cuda, rows, dim, hidden):
    g = gen(rows * 5 + dim + hidden)
    x = _uniform((rows, dim), -1.0, 1.0, g)
    wg = _uniform((dim, hidden), -0.05, 0.05, g)
    wu = _uniform((dim, hidden), -0.05, 0.05, g)
    status = ops.DeviceStatus(cuda)
    got = ops.gemm_swiglu(x.to(cuda), wg.to(cuda), wu.to(cuda), status=status)
    assert status.read() == 0
    want = orc.gemm_swiglu(to_np(x), to_np(wg), to_np(wu), threads=8)
    assert orc.worst_error(to_np(got), want) <= BF16_TOL


def test_gemm_swiglu_known_answers(cuda):
    """tests/kernel_tests.cu:164-173 through the GEMM: x = e0 makes gate and up the
    first weight rows, so the outputs are silu({-1000, -100, 0, 100, 1000}) * 2."""
    gate = torch.zeros(8, 8)
    gate[0, :5] = torch.tensor([-1000.0, -100.0, 0.0, 100.0, 1000.0])
    up = torch.zeros(8, 8)
    up[0, :5] = 2.0
    x = torch.zeros(1, 8)
    x[0, 0] = 1.0
    got = ops.gemm_swiglu(x.to(cuda, torch.bfloat16), gate.to(cuda, torch.bfloat16), up.to(cuda, torch.bfloat16))
    got = got.float().cpu()[0, :5]
    assert torch.isfinite(got).all()
    assert torch.equal(got, torch.tensor([0.0, 0.0, 0.0, 200.0, 2000.0])), got


def test_results_are_deterministic_and_outputs_stay_in_bounds(cuda):
    rows, dim, hidden = 300, 1024, 520
    g = gen(11)
    x = _uniform((rows, dim), -1.0, 1.0, g).to(cuda)
    wg = _uniform((dim, hidden), -0.05, 0.05, g).to(cuda)
    wu = _uniform((dim, hidden), -0.05, 0.05, g).to(cuda)
    # a guard band after the output must survive: the last row block is partial
    buf = torch.full((rows * hidden + 4096,), 7.0, dtype=torch.bfloat16, device=cuda)
    out = buf[: rows * hidden].view(rows, hidden)
    ops.gemm_swiglu(x, wg, wu, out=out)
    first = out.clone()
    ops.gemm_swiglu(x, wg, wu, out=out)
    torch.cuda.synchronize(cuda)
    assert bits_equal(first, out)
    assert torch.all(buf[rows * hidden:] == 7.0)


def test_full_size_prefill_ffn_sampled_rows(cuda):
    """The 8B prefill FFN (32768 tokens, dim 4096, hidden 14336) checked on
    sampled rows: every row block and column block is computed by the same
    code, and rows are independent."""
    rows, dim, hidden = 32768, 4096, 14336
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    x = (torch.randn(rows, dim, device=cuda, generator=g)).to(torch.bfloat16)
    wg = (torch.randn(dim, hidden, device=cuda, generator=g) * 0.02).to(torch.bfloat16)
    wu = (torch.randn(dim, hidden, device=cuda, generator=g) * 0.02).to(torch.bfloat16)
    status = ops.DeviceStatus(cuda)
    out = ops.gemm_swiglu(x, wg, wu, status=status)
    assert status.read() == 0
    sample = torch.tensor([0, 1, 127, 128, 4095, 16384, 25000, rows - 1])
    want = orc.gemm_swiglu(to_np(x[sample.to(cuda)]), to_np(wg), to_np(wu), threads=16)
    assert orc.worst_error(to_np(out[sample.to(cuda)]), want) <= BF16_TOL


def test_fp32_is_refused(cuda):
    a = torch.zeros(16, 16, device=cuda)
    with pytest.raises(_lib.BMError):
        ops.gemm(a, a)

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
    (257, 192, 384),      # wide tile: rows one past a pair block; the 2nd tile's upper column half past the end
    (4097, 512, 288),     # wide tile: 17 pair row blocks (past a tile group of 16); a tile mostly past the columns
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


@pytest.mark.parametrize("m,n,k", [
    (16, 16, 16), (128, 128, 128), (3, 5, 7), (17, 33, 65), (1, 4096, 4096),  # tests/kernel_tests.cu:263-267
    (1, 32000, 288), (1, 288, 288), (1, 768, 288), (1, 288, 768),            # the engine's one-token products
    (7, 300, 200), (9, 130, 4100), (40, 1000, 96),                           # ragged rows, long K, many rows
])
def test_fp32_gemm_matches_the_oracle(cuda, m, n, k):
    """fp32 (the reference's launch_gemm path): CUDA cores, any shape, within 1e-5."""
    g = gen(m + 3 * n + 7 * k)
    a = torch.rand(m, k, generator=g) * 2 - 1
    b = torch.rand(k, n, generator=g) * 2 - 1
    c = torch.full((m, n), float("nan"), device=cuda)
    ops.launch_gemm(c, a.to(cuda), b.to(cuda), m, n, k)
    torch.cuda.synchronize(cuda)
    want = orc.gemm(a.numpy(), b.numpy(), threads=8)
    assert orc.worst_error(c.cpu().numpy(), want) <= 1e-5
    again = ops.gemm(a.to(cuda), b.to(cuda))  # deterministic: the cluster adds its partials in a fixed order
    assert torch.equal(again.cpu(), c.cpu())


def test_fp32_gemm_misaligned_operands(cuda):
    """Rows of B that are not 16-byte multiples, and a B that starts off a 16-byte boundary."""
    g = gen(5)
    m, n, k = 4, 129, 77
    a = (torch.rand(m, k, generator=g) * 2 - 1).to(cuda)
    store = (torch.rand(k * n + 1, generator=g) * 2 - 1).to(cuda)
    b = store[1:].view(k, n)
    c = torch.empty(m, n, device=cuda)
    ops.launch_gemm(c, a, b, m, n, k)
    torch.cuda.synchronize(cuda)
    want = orc.gemm(a.cpu().numpy(), b.cpu().numpy().copy())
    assert orc.worst_error(c.cpu().numpy(), want) <= 1e-5


@pytest.mark.parametrize("rows,dim,hidden", [
    (1, 288, 768), (48, 288, 768),         # the engine's FFN: one token, and a 48-token prompt
    (5, 7, 13), (9, 130, 200), (1, 4096, 14336),  # ragged shapes (hidden % 4 != 0: scalar loads), long rows
    (64, 512, 1000),                        # many rows: the SwiGLU tiles 4 rows, the plain GEMM 8
])
def test_fp32_gemm_swiglu_matches_the_oracle_and_the_unfused_ops(cuda, rows, dim, hidden):
    """bm_gemm_swiglu in fp32: within 1e-5 of the oracle (silu(x Wg) * (x Wu) in double),
    and bit-identical to bm_gemm twice followed by bm_swiglu. Weights at the scale of a
    model's (about 1/sqrt(dim)), so the products stay O(1) at every K."""
    g = gen(rows * 7 + dim + hidden)
    x = (torch.rand(rows, dim, generator=g) * 2 - 1)
    scale = 2.0 / dim ** 0.5
    wg = (torch.rand(dim, hidden, generator=g) * 2 - 1) * scale
    wu = (torch.rand(dim, hidden, generator=g) * 2 - 1) * scale
    xd, wgd, wud = x.to(cuda), wg.to(cuda), wu.to(cuda)
    out = ops.gemm_swiglu(xd, wgd, wud)
    unfused = ops.swiglu(ops.gemm(xd, wgd), ops.gemm(xd, wud))
    torch.cuda.synchronize(cuda)
    want = orc.gemm_swiglu(x.numpy(), wg.numpy(), wu.numpy(), threads=8)
    assert orc.worst_error(out.cpu().numpy(), want) <= 1e-5
    assert bits_equal(out, unfused)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("m,k,widths", [
    (1, 288, (288, 288, 288)),      # the engine's Q, K and V (heads = kv heads)
    (1, 4096, (4096, 1024, 1024)),  # Llama-3-8B Q, K, V (GQA)
    (48, 288, (288, 96, 96)),       # a prompt of 48 tokens, GQA widths
    (3, 64, (40, 0, 24)),           # an empty product between two others
    (2, 256, (128,)),               # one product
])
def test_shared_a_products_match_the_oracle(cuda, dt, m, k, widths):
    """bm_gemm_shared_a: each c[o] = a . b[o] within the GEMM tolerance of its dtype;
    fp32 runs all products in one launch."""
    if dt == torch.bfloat16 and any(w % 8 for w in widths):
        pytest.skip("bf16 widths are multiples of 8")
    g = gen(m + k + sum(widths))
    a = torch.rand(m, k, generator=g) * 2 - 1
    bs = [(torch.rand(k, w, generator=g) * 2 - 1) * 0.2 for w in widths]
    outs = ops.gemm_shared_a(a.to(cuda).to(dt), [b.to(cuda).to(dt) for b in bs])
    torch.cuda.synchronize(cuda)
    tol = 1e-5 if dt == torch.float32 else BF16_TOL
    for b, out in zip(bs, outs):
        assert out.shape == (m, b.shape[1])
        if b.shape[1] == 0:
            continue
        want = orc.gemm(to_np(a.to(dt)), to_np(b.to(dt)), threads=8)
        assert orc.worst_error(to_np(out), want) <= tol


@pytest.mark.parametrize("size,vectors,stride,lo,hi", [
    (1, 1, 1, -4, 4), (100, 1, 100, -4, 4), (4096, 1, 4096, -4, 4),   # tests/kernel_tests.cu:268-275
    (1000, 1, 1000, 995, 1005),                                         # values near 1000 (:140-147)
    (37, 5, 50, -4, 4),                                                 # batch with gaps (:149-160)
    (32000, 3, 32000, -20, 20), (128256, 1, 128256, -10, 10),          # vocab-sized rows
])
def test_softmax_matches_the_oracle(cuda, size, vectors, stride, lo, hi):
    g = gen(size + vectors)
    x = torch.rand((vectors - 1) * stride + size, generator=g) * (hi - lo) + lo
    xd = x.to(cuda)
    ops.launch_softmax_batch(xd, size, vectors, stride)
    torch.cuda.synchronize(cuda)
    want = orc.softmax(x.numpy(), size, vectors, stride)
    assert orc.worst_error(xd.cpu().numpy(), want) <= 1e-5
    for v in range(vectors - 1):  # the gaps between vectors are untouched
        gap = slice(v * stride + size, (v + 1) * stride)
        assert torch.equal(xd.cpu()[gap], x[gap])


def test_softmax_bf16(cuda):
    g = gen(3)
    x = (torch.randn(4, 1000, generator=g) * 3).to(torch.bfloat16)
    xd = x.to(cuda)
    ops.softmax(xd.view(-1), 1000, 4, 1000)
    torch.cuda.synchronize(cuda)
    want = orc.softmax(to_np(x).ravel(), 1000, 4, 1000)
    assert orc.worst_error(to_np(xd).ravel(), want) <= 1e-2

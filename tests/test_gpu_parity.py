"""Parity of the sm_100a kernels with the CPU oracle, through the C ABI.

Each case draws seeded inputs with the shapes of one workload (tiny Llama
layer, Llama-3-8B decode and prefill, SwiGLU stress, Llama-3-70B; rows reduced
where the oracle needs them to finish in seconds), runs the kernel on cuda:0
and compares with the oracle (the reference's double-precision check loops):
fp32 within 1e-5 and bf16 within 1e-2 in the reference's metric
|got - want| / (1 + |want|); gather and KV-cache copies bit-exact.
"""
import numpy as np
import pytest
import torch

from baremetalinferenceengine_b200 import ops
from baremetalinferenceengine_b200._lib import BM_DEVERR_BAD_ID, BM_DEVERR_BAD_POSITION, BM_DEVERR_BAD_SEQUENCE, BMError
from oracle import oracle as orc
from tests.helpers import TOL, bits_equal, from_np, gen, randn, to_np

pytestmark = pytest.mark.gpu

# name: (rows, dim, hq, hkv, hd, ffn, vocab, theta, max_seq, num_seqs)
SHAPES = {
    "tinyllama": (256, 288, 6, 6, 48, 768, 32000, 1e4, 256, 1),
    "llama8b_decode": (64, 4096, 32, 8, 128, 14336, 128256, 5e5, 8192, 64),
    "llama8b_prefill": (384, 4096, 32, 8, 128, 14336, 128256, 5e5, 8192, 4),
    "llama70b": (96, 8192, 64, 8, 128, 28672, 128256, 5e5, 8192, 16),
}
DTYPES = [torch.float32, torch.bfloat16]
CASES = [(n, dt) for n in SHAPES for dt in DTYPES if not (n == "tinyllama" and dt == torch.bfloat16)]


def case_id(c):
    return f"{c[0]}-{str(c[1]).split('.')[-1]}"


def worst(got: torch.Tensor, want: np.ndarray) -> float:
    return orc.worst_error(to_np(got), want)


def positions_for(name, rows, max_seq, num_seqs, g):
    """Token positions and sequence ids the way each workload lays them out."""
    if name == "tinyllama":
        pos = torch.arange(rows, dtype=torch.int32)
        seq = torch.zeros(rows, dtype=torch.int32)
    elif name == "llama8b_decode":
        pos = torch.randint(0, max_seq, (rows,), generator=g, dtype=torch.int32)
        seq = torch.arange(rows, dtype=torch.int32) % num_seqs
    else:  # prefill-shaped: positions tile each sequence; sample spread over all positions
        per = rows // num_seqs
        pos = torch.cat([torch.linspace(0, max_seq - 1, per).round().to(torch.int32) for _ in range(num_seqs)])
        seq = torch.arange(num_seqs, dtype=torch.int32).repeat_interleave(per)
    return pos, seq


# ----------------------------------------------------------------------------- gather

def device_table(vocab, dim, dt, device, seed):
    """N(0, 0.02) embedding table drawn on the device (a 128256-row table is GBs)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return (torch.randn(vocab, dim, generator=g, device=device) * 0.02).to(dt)


@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_embed_gather(cuda, case):
    name, dt = case
    rows, dim, *_, vocab, _, _, _ = SHAPES[name]
    g = gen(1)
    table = device_table(vocab, dim, dt, cuda, seed=1)
    ids = torch.randint(0, vocab, (rows,), generator=g, dtype=torch.int32)
    ids[-1] = vocab - 1  # the last row of the table: the largest byte offset
    out = ops.embed_gather(table, ids.to(cuda))
    want, bad = orc.gather(to_np(table), ids.numpy())
    assert bad == 0
    assert bits_equal(out, from_np(want))


def test_embed_gather_zipf_repeats(cuda):
    """Zipf(1.1) ids over 128256 (the SwiGLU-stress gather): heavy repeats, bit-exact."""
    rng = np.random.default_rng(4)
    vocab, dim, rows = 128256, 4096, 4096
    p = 1.0 / np.arange(1, vocab + 1) ** 1.1
    ids = rng.choice(vocab, size=rows, p=p / p.sum()).astype(np.int32)
    table = device_table(vocab, dim, torch.bfloat16, cuda, seed=5)
    out = ops.embed_gather(table, torch.from_numpy(ids).to(cuda))
    want, _ = orc.gather(to_np(table), ids)
    assert bits_equal(out, from_np(want))


@pytest.mark.parametrize("dt", DTYPES, ids=["f32", "bf16"])
def test_embed_gather_bad_ids_leave_rows_and_flag(cuda, dt):
    vocab, dim = 100, 64
    table = randn((vocab, dim), dt, gen(2))
    ids = torch.tensor([3, -1, 99, 100, 7, 2**31 - 1], dtype=torch.int32)
    sentinel = torch.full((ids.numel(), dim), 7.0, dtype=dt)
    out = sentinel.clone().to(cuda)
    status = ops.DeviceStatus(cuda)
    ops.embed_gather(table.to(cuda), ids.to(cuda), out=out, status=status)
    assert status.read() == BM_DEVERR_BAD_ID
    assert status.read() == 0  # read clears
    out = out.cpu()
    for r, i in enumerate(ids.tolist()):
        assert bits_equal(out[r], table[i] if 0 <= i < vocab else sentinel[r])


@pytest.mark.parametrize("dt", DTYPES, ids=["f32", "bf16"])
@pytest.mark.parametrize("dim", [1, 3, 288, 301])
def test_embed_gather_ragged_and_strided(cuda, dt, dim):
    """Odd dims and an out pitch of dim+1 take the scalar path; results are the same."""
    vocab, rows = 50, 17
    table = randn((vocab, dim), dt, gen(dim), 1.0)
    ids = torch.randint(0, vocab, (rows,), generator=gen(3), dtype=torch.int32)
    big = torch.zeros(rows, dim + 1, dtype=dt, device=cuda)
    ops.embed_gather(table.to(cuda), ids.to(cuda), out=big[:, :dim])
    assert bits_equal(big[:, :dim], table[ids.long()])
    assert bits_equal(big[:, dim:], torch.zeros(rows, 1, dtype=dt))


def test_embed_gather_empty(cuda):
    table = torch.zeros(10, 8, device=cuda)
    out = ops.embed_gather(table, torch.zeros(0, dtype=torch.int32, device=cuda))
    assert out.shape == (0, 8)


# ----------------------------------------------------------------------------- RMSNorm

@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_rmsnorm(cuda, case):
    name, dt = case
    rows, dim = SHAPES[name][:2]
    g = gen(10)
    x = randn((rows, dim), dt, g)
    w = randn((dim,), dt, g, 0.02, 1.0)
    out = ops.rmsnorm(x.to(cuda), w.to(cuda))
    assert worst(out, orc.rmsnorm(to_np(x), to_np(w))) <= TOL[dt]


@pytest.mark.parametrize("size", [64, 256, 300, 4096])
def test_rmsnorm_reference_sizes(cuda, size):
    """The reference's rms_norm cases (tests/kernel_tests.cu:268-271): one vector,
    inputs U[-1,1], weights U[0.5,1.5]."""
    g = gen(size)
    x = torch.rand(1, size, generator=g) * 2 - 1
    w = torch.rand(size, generator=g) + 0.5
    out = ops.rmsnorm(x.to(cuda), w.to(cuda))
    assert worst(out, orc.rmsnorm(x.numpy(), w.numpy())) <= 1e-5


@pytest.mark.parametrize("dt", DTYPES, ids=["f32", "bf16"])
@pytest.mark.parametrize("rows,dim", [(1, 1), (3, 7), (17, 300), (5, 1000), (2, 8192 * 8 + 8), (4, 40000)])
def test_rmsnorm_ragged_and_wide(cuda, dt, rows, dim):
    g = gen(rows * 7 + dim)
    x = randn((rows, dim), dt, g)
    w = randn((dim,), dt, g, 0.02, 1.0)
    out = ops.rmsnorm(x.to(cuda), w.to(cuda))
    assert worst(out, orc.rmsnorm(to_np(x), to_np(w))) <= TOL[dt]


@pytest.mark.parametrize("dt", DTYPES, ids=["f32", "bf16"])
def test_rmsnorm_in_place(cuda, dt):
    """ExecutionEngine::forward normalises in place (tests/kernel_tests.cu:88-103)."""
    g = gen(11)
    x = randn((33, 4096), dt, g)
    w = randn((4096,), dt, g, 0.02, 1.0)
    want = orc.rmsnorm(to_np(x), to_np(w))
    xd = x.to(cuda)
    ops.rmsnorm(xd, w.to(cuda), out=xd)
    assert worst(xd, want) <= TOL[dt]


def test_rmsnorm_strided_rows(cuda):
    g = gen(12)
    base = randn((9, 4096 + 64), torch.bfloat16, g)
    w = randn((4096,), torch.bfloat16, g, 0.02, 1.0)
    xv = base.to(cuda)[:, :4096]
    out = ops.rmsnorm(xv, w.to(cuda))
    assert worst(out, orc.rmsnorm(to_np(base[:, :4096]), to_np(w))) <= 1e-2


def test_rmsnorm_rejects_partial_overlap(cuda):
    x = torch.randn(4, 64, device=cuda)
    w = torch.ones(64, device=cuda)
    flat = x.view(-1)
    with pytest.raises(BMError):
        ops.rmsnorm(flat[:192].view(3, 64), w, out=flat[64:].view(3, 64))


# ----------------------------------------------------------------------------- add + RMSNorm

@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_add_rmsnorm(cuda, case):
    name, dt = case
    rows, dim = SHAPES[name][:2]
    g = gen(20)
    h = randn((rows, dim), dt, g)
    p = randn((rows, dim), dt, g)
    w = randn((dim,), dt, g, 0.02, 1.0)
    hd_, pd = h.to(cuda), p.to(cuda)
    y = ops.add_rmsnorm(hd_, pd, w.to(cuda))
    want_h, want_y = orc.add_rmsnorm(to_np(h), to_np(p), to_np(w))
    assert bits_equal(hd_, from_np(want_h))  # the residual is an fp32 add, rounded once: exact
    assert worst(y, want_y) <= TOL[dt]
    assert bits_equal(pd, p)  # delta untouched


@pytest.mark.parametrize("dt", DTYPES, ids=["f32", "bf16"])
@pytest.mark.parametrize("rows,dim", [(1, 8), (3, 300), (7, 1001)])
def test_add_rmsnorm_ragged(cuda, dt, rows, dim):
    g = gen(21 + dim)
    h, p = randn((rows, dim), dt, g), randn((rows, dim), dt, g)
    w = randn((dim,), dt, g, 0.02, 1.0)
    hd_ = h.to(cuda)
    y = ops.add_rmsnorm(hd_, p.to(cuda), w.to(cuda))
    want_h, want_y = orc.add_rmsnorm(to_np(h), to_np(p), to_np(w))
    assert bits_equal(hd_, from_np(want_h))
    assert worst(y, want_y) <= TOL[dt]


# ----------------------------------------------------------------------------- add

@pytest.mark.parametrize("dt", DTYPES, ids=["f32", "bf16"])
@pytest.mark.parametrize("n", [1, 1000, 4099, 1 << 20])
def test_add_in_place(cuda, dt, n):
    """The reference's add case is in place (tests/kernel_tests.cu:202-212)."""
    g = gen(n)
    a, b = randn((n,), dt, g), randn((n,), dt, g)
    ad = a.to(cuda)
    ops.add(ad, b.to(cuda), out=ad)
    assert bits_equal(ad, from_np(orc.add(to_np(a), to_np(b))))


# ----------------------------------------------------------------------------- SwiGLU

@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_swiglu(cuda, case):
    name, dt = case
    rows, ffn = SHAPES[name][0], SHAPES[name][5]
    g = gen(30)
    gate, up = randn((rows, ffn), dt, g), randn((rows, ffn), dt, g)
    out = ops.swiglu(gate.to(cuda), up.to(cuda))
    assert worst(out, orc.swiglu(to_np(gate), to_np(up))) <= TOL[dt]


@pytest.mark.parametrize("dt", DTYPES, ids=["f32", "bf16"])
def test_swiglu_stress_outliers(cuda, dt):
    """SwiGLU stress shape (FFN 14336) with 1% of entries at +-20 to exercise saturation."""
    rows, ffn = 128, 14336
    g = gen(31)
    gate, up = randn((rows, ffn), torch.float32, g), randn((rows, ffn), torch.float32, g)
    for t in (gate, up):
        mask = torch.rand(t.shape, generator=g) < 0.01
        t[mask] = torch.where(torch.rand(t.shape, generator=g) < 0.5, -20.0, 20.0)[mask]
    gate, up = gate.to(dt), up.to(dt)
    out = ops.swiglu(gate.to(cuda), up.to(cuda))
    assert worst(out, orc.swiglu(to_np(gate), to_np(up))) <= TOL[dt]


@pytest.mark.parametrize("dt", DTYPES, ids=["f32", "bf16"])
def test_swiglu_known_answers(cuda, dt):
    """Known answers of tests/kernel_tests.cu:164-173: silu saturates, stays finite."""
    gate = torch.tensor([-1000.0, -100.0, 0.0, 100.0, 1000.0], dtype=dt)
    up = torch.full((5,), 2.0, dtype=dt)
    out = ops.swiglu(gate.to(cuda), up.to(cuda)).float().cpu()
    want = torch.tensor([0.0, 0.0, 0.0, 200.0, 2000.0])
    assert torch.isfinite(out).all()
    assert ((out - want).abs() / (1 + want.abs())).max().item() <= TOL[dt]


@pytest.mark.parametrize("dt", DTYPES, ids=["f32", "bf16"])
@pytest.mark.parametrize("n", [1, 3, 4097, 4099])
def test_swiglu_tails_and_unaligned(cuda, dt, n):
    g = gen(32 + n)
    gate, up = randn((n + 1,), dt, g), randn((n + 1,), dt, g)
    gd, ud = gate.to(cuda), up.to(cuda)
    out = torch.zeros(n + 1, dtype=dt, device=cuda)
    ops.swiglu(gd[:n], ud[:n], out=out[:n])  # aligned, ragged tail
    assert worst(out[:n], orc.swiglu(to_np(gate[:n]), to_np(up[:n]))) <= TOL[dt]
    ops.swiglu(gd[1:], ud[1:], out=out[1:])  # every pointer 1 element off: scalar path
    assert worst(out[1:], orc.swiglu(to_np(gate[1:]), to_np(up[1:]))) <= TOL[dt]


# ----------------------------------------------------------------------------- RoPE + KV cache

def _rope_case(name, dt, seed=40):
    rows, dim, hq, hkv, hd, ffn, vocab, theta, max_seq, num_seqs = SHAPES[name]
    g = gen(seed)
    q = randn((rows, hq, hd), dt, g)
    k = randn((rows, hkv, hd), dt, g)
    v = randn((rows, hkv, hd), dt, g)
    pos, seq = positions_for(name, rows, max_seq, num_seqs, g)
    cache_shape = (num_seqs, hkv, max_seq, hd)
    kc = torch.full(cache_shape, -3.0, dtype=dt)  # sentinel: untouched slots must keep it
    vc = torch.full(cache_shape, 5.0, dtype=dt)
    return q, k, v, pos, seq, kc, vc, theta, max_seq


@pytest.mark.parametrize("use_table", [True, False], ids=["table", "fp64"])
@pytest.mark.parametrize("case", CASES, ids=case_id)
def test_rope_kv_store(cuda, case, use_table):
    name, dt = case
    q, k, v, pos, seq, kc, vc, theta, max_seq = _rope_case(name, dt)
    qd, kd, vd, kcd, vcd = (t.to(cuda) for t in (q, k, v, kc, vc))
    table = ops.RopeTable(max_seq, q.shape[2], theta, cuda) if use_table else None
    status = ops.DeviceStatus(cuda)
    ops.rope_kv_store(qd, kd, vd, pos.to(cuda), kcd, vcd, table=table, theta=theta, seq_ids=seq.to(cuda),
                      status=status)
    assert status.read() == 0
    want_q, want_kc, want_vc, bad = orc.rope_kv_store(to_np(q), to_np(k), to_np(v), pos.numpy(), to_np(kc),
                                                      to_np(vc), theta, seq_ids=seq.numpy())
    assert bad == 0
    assert worst(qd, want_q) <= TOL[dt]
    assert worst(kcd, want_kc) <= TOL[dt]
    assert bits_equal(vcd, from_np(want_vc))  # v is a copy: exact, and sentinels survive
    # untouched K slots keep the sentinel bit for bit
    written = torch.zeros(kc.shape[0], kc.shape[2], dtype=torch.bool)
    written[seq.long(), pos.long()] = True
    kcc = kcd.cpu()
    assert bits_equal(kcc.permute(0, 2, 1, 3)[~written], kc.permute(0, 2, 1, 3)[~written])
    assert bits_equal(kd, k) and bits_equal(vd, v)  # k and v inputs are not modified


@pytest.mark.parametrize("use_table", [True, False], ids=["table", "fp64"])
@pytest.mark.parametrize("dt", DTYPES, ids=["f32", "bf16"])
@pytest.mark.parametrize("rows,hq,hkv,hd", [(512, 6, 6, 48), (1024, 32, 8, 128), (600, 64, 8, 128), (700, 5, 1, 6),
                                            (513, 4, 2, 34), (512, 2, 1, 1024)])
def test_rope_kv_store_large_batches(cuda, use_table, dt, rows, hq, hkv, hd):
    """Batches of >= 512 tokens take the warp-per-token kernel (heads spread over the
    lanes, cos/sin kept in registers); head_dim 1024 falls back to one block per token."""
    max_seq, num_seqs = 2048, 3
    g = gen(rows + hq + hd)
    q, k, v = randn((rows, hq, hd), dt, g), randn((rows, hkv, hd), dt, g), randn((rows, hkv, hd), dt, g)
    perm = torch.randperm(num_seqs * max_seq, generator=g)[:rows]
    pos, seq = (perm % max_seq).to(torch.int32), (perm // max_seq).to(torch.int32)
    kc = torch.full((num_seqs, hkv, max_seq, hd), -3.0, dtype=dt)
    vc = torch.full((num_seqs, hkv, max_seq, hd), 5.0, dtype=dt)
    qd, kcd, vcd = q.to(cuda), kc.to(cuda), vc.to(cuda)
    table = ops.RopeTable(max_seq, hd, 5e5, cuda) if use_table else None
    ops.rope_kv_store(qd, k.to(cuda), v.to(cuda), pos.to(cuda), kcd, vcd, table=table, theta=5e5,
                      seq_ids=seq.to(cuda))
    want_q, want_kc, want_vc, _ = orc.rope_kv_store(to_np(q), to_np(k), to_np(v), pos.numpy(), to_np(kc), to_np(vc),
                                                    5e5, seq_ids=seq.numpy())
    assert worst(qd, want_q) <= TOL[dt]
    assert worst(kcd, want_kc) <= TOL[dt]
    assert bits_equal(vcd, from_np(want_vc))
    # the in-place variant and the plain store at the same sizes
    qd2, kd2 = q.to(cuda), k.to(cuda)
    ops.rope(qd2, kd2, pos.to(cuda), table=table, theta=5e5)
    assert worst(qd2, orc.rope(to_np(q), pos.numpy(), 5e5)) <= TOL[dt]
    assert worst(kd2, orc.rope(to_np(k), pos.numpy(), 5e5)) <= TOL[dt]
    vcd2 = vc.to(cuda)
    ops.kv_store(vcd2, v.to(cuda), pos.to(cuda), seq.to(cuda))
    assert bits_equal(vcd2, from_np(want_vc))


@pytest.mark.parametrize("dt", DTYPES, ids=["f32", "bf16"])
@pytest.mark.parametrize("table_len,hd", [(1000, 128), (8192, 128), (256, 48), (3, 64)])
def test_rope_on_chip_table_boundaries(cuda, dt, table_len, hd):
    """Batches of >= 512 tokens with a table take (cos, sin) from the on-chip table:
    fine rows 0..L-1 and coarse rows 0, L, 2L, ... in shared memory, combined by angle
    addition. Positions on both sides of every L boundary, the last table row, and
    position 0, for a table length that is not a power of two as well: within the
    tolerance of the double-precision oracle, and position 0 exactly the identity."""
    rows, hq, hkv = 1024, 8, 2
    g = gen(table_len + hd)
    lg = min(range(0, 31), key=lambda e: (-(-table_len // 2**e) + 2**e) if 2**e <= table_len else 1 << 40)
    L = 2 ** lg
    edge = sorted({p for b in range(0, table_len, L) for p in (b - 1, b, b + 1) if 0 <= p < table_len}
                  | {0, table_len - 1})
    pos = torch.tensor((edge * (rows // len(edge) + 1))[:rows], dtype=torch.int32)
    pos[:8] = 0
    q, k = randn((rows, hq, hd), dt, g), randn((rows, hkv, hd), dt, g)
    table = ops.RopeTable(table_len, hd, 5e5, cuda)
    qd, kd = q.to(cuda), k.to(cuda)
    status = ops.DeviceStatus(cuda)
    ops.rope(qd, kd, pos.to(cuda), table=table, status=status)
    assert status.read() == 0
    assert worst(qd, orc.rope(to_np(q), pos.numpy(), 5e5)) <= TOL[dt]
    assert worst(kd, orc.rope(to_np(k), pos.numpy(), 5e5)) <= TOL[dt]
    assert bits_equal(qd[:8], q[:8])  # position 0: the identity, bit for bit
    # the fused form (K into the cache): the edge positions repeated, each repetition
    # in its own sequence, so every (sequence, position) slot is written once
    fpos = torch.tensor((edge * (rows // len(edge) + 1))[:rows], dtype=torch.int32)
    seq = torch.arange(rows, dtype=torch.int32) // len(edge)
    v = randn((rows, hkv, hd), dt, g)
    kc = torch.zeros(int(seq.max()) + 1, hkv, table_len, hd, dtype=dt)
    qd, kcd, vcd = q.to(cuda), kc.to(cuda), kc.clone().to(cuda)
    ops.rope_kv_store(qd, k.to(cuda), v.to(cuda), fpos.to(cuda), kcd, vcd, table=table, seq_ids=seq.to(cuda),
                      status=status)
    assert status.read() == 0
    want_q, want_kc, _, bad = orc.rope_kv_store(to_np(q), to_np(k), to_np(v), fpos.numpy(), to_np(kc), to_np(kc),
                                                5e5, seq_ids=seq.numpy())
    assert bad == 0
    assert worst(qd, want_q) <= TOL[dt]
    assert worst(kcd, want_kc) <= TOL[dt]


@pytest.mark.parametrize("dt", DTYPES, ids=["f32", "bf16"])
@pytest.mark.parametrize("hq,hkv,hd", [(6, 6, 48), (6, 3, 48), (8, 8, 128), (5, 1, 6), (4, 2, 34)])
def test_rope_in_place(cuda, dt, hq, hkv, hd):
    """Batched launch_rope, incl. the reference's GQA-shaped case (6/3 heads) and
    head dims whose halves are not vector multiples (scalar path)."""
    rows = 19
    g = gen(hq * 100 + hd)
    q, k = randn((rows, hq, hd), dt, g), randn((rows, hkv, hd), dt, g)
    pos = torch.randint(0, 4096, (rows,), generator=g, dtype=torch.int32)
    qd, kd = q.to(cuda), k.to(cuda)
    ops.rope(qd, kd, pos.to(cuda), theta=1e4)
    assert worst(qd, orc.rope(to_np(q), pos.numpy(), 1e4)) <= TOL[dt]
    assert worst(kd, orc.rope(to_np(k), pos.numpy(), 1e4)) <= TOL[dt]


def test_rope_position_zero_is_identity(cuda):
    """tests/kernel_tests.cu:280: at position 0 the rotation is exactly the identity."""
    q = torch.randn(3, 6, 48)
    qd = q.to(cuda)
    ops.rope(qd[:1], None, 0, theta=1e4)  # one token at pos0 = 0 (fp64 cos/sin)
    ops.rope(qd, None, torch.zeros(3, dtype=torch.int32, device=cuda), table=ops.RopeTable(8, 48, 1e4, cuda))
    assert bits_equal(qd, q)
    ops.rope(qd, None, 0, theta=1e4)  # pos0 = 0 over 3 tokens means positions 0, 1, 2
    want = orc.rope(q.numpy(), np.arange(3, dtype=np.int32), 1e4)
    assert bits_equal(qd[0], q[0]) and worst(qd, want) <= 1e-5


def test_rope_bad_positions_and_sequences_flag_and_skip(cuda):
    rows, hq, hkv, hd, max_seq, num_seqs = 6, 4, 2, 64, 16, 2
    q, k, v = torch.randn(rows, hq, hd), torch.randn(rows, hkv, hd), torch.randn(rows, hkv, hd)
    pos = torch.tensor([0, 15, 16, -1, 3, 4], dtype=torch.int32)
    seq = torch.tensor([0, 1, 0, 0, 2, -1], dtype=torch.int32)
    kc = torch.full((num_seqs, hkv, max_seq, hd), 9.0)
    vc = torch.full((num_seqs, hkv, max_seq, hd), 9.0)
    qd, kcd, vcd = q.to(cuda), kc.to(cuda), vc.to(cuda)
    status = ops.DeviceStatus(cuda)
    table = ops.RopeTable(max_seq, hd, 1e4, cuda)
    ops.rope_kv_store(qd, k.to(cuda), v.to(cuda), pos.to(cuda), kcd, vcd, table=table, theta=1e4,
                      seq_ids=seq.to(cuda), status=status)
    assert status.read() == BM_DEVERR_BAD_POSITION | BM_DEVERR_BAD_SEQUENCE
    want_q, want_kc, want_vc, bad = orc.rope_kv_store(q.numpy(), k.numpy(), v.numpy(), pos.numpy(), kc.numpy(),
                                                      vc.numpy(), 1e4, seq_ids=seq.numpy(), table_len=max_seq)
    assert bad == BM_DEVERR_BAD_POSITION | BM_DEVERR_BAD_SEQUENCE
    qc = qd.cpu()
    for r in (2, 3, 4, 5):  # skipped rows: q untouched
        assert bits_equal(qc[r], q[r])
    assert worst(qd, want_q) <= 1e-5
    assert worst(kcd, want_kc) <= 1e-5
    assert bits_equal(vcd, from_np(want_vc))


def test_rope_beyond_table_is_flagged(cuda):
    q = torch.randn(2, 2, 8)
    qd = q.to(cuda)
    status = ops.DeviceStatus(cuda)
    ops.rope(qd, None, torch.tensor([3, 4], dtype=torch.int32, device=cuda), table=ops.RopeTable(4, 8, 1e4, cuda),
             status=status)
    assert status.read() == BM_DEVERR_BAD_POSITION
    assert bits_equal(qd.cpu()[1], q[1])


@pytest.mark.parametrize("dt", DTYPES, ids=["f32", "bf16"])
def test_kv_store(cuda, dt):
    rows, h, hd, max_seq, num_seqs = 40, 8, 128, 64, 3
    g = gen(50)
    src = randn((rows, h, hd), dt, g)
    pos = torch.randint(0, max_seq, (rows,), generator=g, dtype=torch.int32)
    seq = torch.randint(0, num_seqs, (rows,), generator=g, dtype=torch.int32)
    # distinct (seq, pos) pairs so that the result does not depend on write order
    key = seq.long() * max_seq + pos.long()
    keep = torch.ones(rows, dtype=torch.bool)
    seen = set()
    for i, kk in enumerate(key.tolist()):
        keep[i] = kk not in seen
        seen.add(kk)
    src, pos, seq = src[keep], pos[keep], seq[keep]
    cache = randn((num_seqs, h, max_seq, hd), dt, g)
    cd = cache.to(cuda)
    ops.kv_store(cd, src.to(cuda), pos.to(cuda), seq.to(cuda))
    want, bad = orc.kv_store(to_np(cache), to_np(src), pos.numpy(), seq.numpy())
    assert bad == 0
    assert bits_equal(cd, from_np(want))


def test_kv_store_reference_case(cuda):
    """tests/kernel_tests.cu:214-227: 3 heads, hd 8, max_seq 5, pos 2 — one position
    written, the rest left alone."""
    g = gen(51)
    cache = torch.rand(1, 3, 5, 8, generator=g) * 2 - 1
    src = torch.rand(1, 3, 8, generator=g) * 2 - 1
    cd = cache.to(cuda)
    ops.kv_store(cd, src.to(cuda), 2)
    want, _ = orc.kv_store(cache.numpy(), src.numpy(), 2)
    assert bits_equal(cd, from_np(want))


def test_rope_table_matches_oracle(cuda):
    for max_pos, hd, theta in [(256, 48, 1e4), (8192, 128, 5e5)]:
        t = ops.RopeTable(max_pos, hd, theta, cuda)
        want = orc.rope_table(max_pos, hd, theta)
        got = t.data.cpu().numpy()
        assert np.abs(got - want).max() <= 2e-7  # both round the fp64 value once to fp32


# ----------------------------------------------------------------------------- argument checks

def test_invalid_arguments_raise(cuda):
    x = torch.randn(2, 8, device=cuda)
    with pytest.raises(BMError):
        ops.rmsnorm(x.half(), torch.ones(8, device=cuda).half())
    with pytest.raises(BMError):
        ops.rope(torch.randn(1, 2, 7, device=cuda), None, 0)  # odd head_dim
    with pytest.raises(BMError):
        ops.rope_kv_store(torch.randn(2, 2, 8, device=cuda), torch.randn(2, 1, 8, device=cuda),
                          torch.randn(2, 1, 8, device=cuda), 7, torch.zeros(1, 1, 8, 8, device=cuda),
                          torch.zeros(1, 1, 8, 8, device=cuda))  # pos0 + rows > max_seq

"""Pins the CPU oracle to the reference before it is trusted as the checker.

1. The reference's own test harness (tests/kernel_tests.cu, unmodified, built by
   oracle/Makefile with its launch_* served by the oracle on host memory) grades
   the oracle with the reference's double-precision loops: every layer-op check
   must pass at worst error 0 (bit-identical float outputs).
2. The oracle's RoPE equals the reference's reference_rope bit for bit at many
   positions, head dims, head counts and both thetas (libref_cpu.so).
3. The committed golden fixtures (made from the reference's code by
   tests/golden/make_golden.py) and the reference's known answers.
4. Oracle-internal properties (bf16 rounding against torch, row independence,
   in-place semantics, bad-row handling).
"""
import os
import re
import subprocess

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests.helpers import from_np, reference_dir, to_np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _ensure_ref():
    """Builds oracle/_ref from the reference's sources when they are present."""
    ref = reference_dir()
    if not orc.ref_available() and ref is not None:
        subprocess.run(["make", "-s", "-C", os.path.dirname(orc.__file__), "ref", f"REF={ref}"], check=True)
    if not orc.ref_available():
        pytest.skip("oracle/_ref is not built and the reference's sources are absent")


IN_SCOPE = ("rms_norm", "swiglu", "rope", "add in place", "kv store")


def test_reference_harness_grades_the_oracle():
    _ensure_ref()
    proc = subprocess.run([orc.REF_HARNESS_CPU], capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    lines = [l for l in proc.stdout.splitlines() if l.startswith(("PASS", "FAIL"))]
    scoped = [l for l in lines if any(l[6:].startswith(s) for s in IN_SCOPE)]
    assert len(scoped) == 15, scoped  # 5 rms_norm, 2 swiglu, 6 rope, add, kv store: kernel_tests.cu:268-284
    for line in scoped:
        assert line.startswith("PASS"), line
        err = float(re.search(r"worst relative error (\S+)", line).group(1))
        # exact everywhere except the known-answer test, whose want rounds silu(-100)*2 (~7e-42) to 0
        assert err == 0.0 or ("stays finite" in line and err < 1e-40), line
    softmax = [l for l in lines if l[6:].startswith("softmax")]
    assert len(softmax) == 5, softmax  # kernel_tests.cu: sizes 1, 100, 4096, near 1000, batch with gaps
    for line in softmax:
        assert line.startswith("PASS") and float(re.search(r"worst relative error (\S+)", line).group(1)) == 0.0, line
    gemm = [l for l in lines if l[6:].startswith("gemm")]
    assert len(gemm) == 5, gemm  # kernel_tests.cu:263-267, served by oracle_gemm
    for line in gemm:
        assert line.startswith("PASS") and float(re.search(r"worst relative error (\S+)", line).group(1)) == 0.0, line


@pytest.mark.parametrize("theta", [1e4, 5e5])
@pytest.mark.parametrize("hd,heads", [(48, 6), (48, 3), (128, 8), (128, 32), (64, 2), (6, 1)])
def test_oracle_rope_is_reference_rope(theta, hd, heads):
    _ensure_ref()
    rng = np.random.default_rng(hd * heads)
    positions = [0, 1, 2, 37, 255, 1000, 4095, 8191, 65535]
    x = rng.uniform(-1, 1, size=(len(positions), heads, hd)).astype(np.float32)
    got = orc.rope(x, np.array(positions, np.int32), theta)
    for r, p in enumerate(positions):
        want = orc.ref_reference_rope(x[r], p, theta)
        assert np.array_equal(got[r].view(np.uint32), want.view(np.uint32)), (p, hd, heads)


def test_golden_rope_fixtures():
    z = np.load(os.path.join(GOLDEN, "rope_reference.npz"))
    for n in range(int(z["count"])):
        pos, hd, heads, theta = z[f"meta{n}"]
        got = orc.rope(z[f"x{n}"][None], int(pos), float(theta))[0]
        assert np.array_equal(got.view(np.uint32), z[f"out{n}"].view(np.uint32)), n


def test_golden_swiglu_known_answers():
    z = np.load(os.path.join(GOLDEN, "swiglu_known_answers.npz"))
    for dt in (np.float32, np.uint16):
        g, u = z["gate"], z["up"]
        if dt == np.uint16:
            g, u = orc.f32_to_bf16(g), orc.f32_to_bf16(u)
        got = orc.swiglu(g, u)
        assert orc.worst_error(got, z["want"]) < 1e-30


@pytest.mark.parametrize("m,n,k", [(16, 16, 16), (128, 128, 128), (3, 5, 7), (17, 33, 65), (1, 300, 200)])
def test_oracle_gemm_is_reference_gemm(m, n, k):
    _ensure_ref()
    rng = np.random.default_rng(m * n + k)
    a = rng.uniform(-1, 1, size=(m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, size=(k, n)).astype(np.float32)
    want = orc.ref_reference_gemm(a, b)
    for threads in (1, 4):
        assert np.array_equal(orc.gemm(a, b, threads).view(np.uint32), want.view(np.uint32)), threads


def test_golden_gemm_fixtures():
    z = np.load(os.path.join(GOLDEN, "gemm_reference.npz"))
    for n in range(int(z["count"])):
        a, b = orc.bf16_to_f32(z[f"a{n}"]), orc.bf16_to_f32(z[f"b{n}"])
        assert np.array_equal(orc.gemm(a, b).view(np.uint32), z[f"c{n}"].view(np.uint32)), n
        # in bf16 storage the oracle rounds the same double sums once more, to bf16
        got16 = orc.gemm(z[f"a{n}"], z[f"b{n}"])
        assert np.array_equal(got16, orc.f32_to_bf16(z[f"c{n}"])) or orc.worst_error(got16, z[f"c{n}"]) <= 2.0 ** -8


def test_oracle_gemm_swiglu_is_gemm_then_swiglu():
    z = np.load(os.path.join(GOLDEN, "gemm_reference.npz"))
    x, wg, wu = (orc.bf16_to_f32(z[k]) for k in ("ffn_x", "ffn_w_gate", "ffn_w_up"))
    assert np.array_equal(orc.gemm(x, wg).view(np.uint32), z["ffn_gate"].view(np.uint32))
    assert np.array_equal(orc.gemm(x, wu).view(np.uint32), z["ffn_up"].view(np.uint32))
    fused = orc.gemm_swiglu(x, wg, wu, threads=3)
    # the fused oracle keeps gate and up in double; rounding them to fp32 first moves the result by ~1 ulp
    assert orc.worst_error(fused, orc.swiglu(z["ffn_gate"], z["ffn_up"])) < 1e-6
    # known answers through the GEMM: x = e0, so gate and up are the first weight rows
    gate = np.zeros((8, 8), np.float32)
    gate[0, :5] = [-1000.0, -100.0, 0.0, 100.0, 1000.0]
    up = np.zeros((8, 8), np.float32)
    up[0, :5] = 2.0
    e0 = np.zeros((1, 8), np.float32)
    e0[0, 0] = 1.0
    out = orc.gemm_swiglu(e0, gate, up)
    assert orc.worst_error(out[0, :5], np.array([0.0, 0.0, 0.0, 200.0, 2000.0], np.float32)) < 1e-30


def test_bf16_rounding_matches_torch():
    x = torch.randn(1 << 16) * torch.logspace(-30, 30, 1 << 16)
    x[:4] = torch.tensor([float("inf"), -float("inf"), 0.0, -0.0])
    want = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(orc.f32_to_bf16(x.numpy()), want)
    # the C routine agrees with the vectorised one
    L = orc.lib()
    for v in x[:2048].tolist():
        assert L.oracle_f32_to_bf16(v) == orc.f32_to_bf16(np.array([v], np.float32))[0]


def test_f64_to_bf16_is_single_rounding():
    # 1 + 2^-8 + 2^-30 is above the bf16 midpoint 1 + 2^-8: it rounds up, although
    # a float32 first step (round to nearest) would land on the midpoint and then tie to even (down).
    x = 1.0 + 2.0**-8 + 2.0**-30
    assert orc.lib().oracle_f64_to_bf16(x) == 0x3F81
    assert orc.lib().oracle_f64_to_bf16(1.0 + 2.0**-8) == 0x3F80  # an exact tie: to even


def test_rmsnorm_rows_are_independent_and_in_place_safe():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((5, 300)).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(300)).astype(np.float32)
    full = orc.rmsnorm(x, w)
    for r in range(5):
        assert np.array_equal(orc.rmsnorm(x[r : r + 1], w)[0], full[r])
    # a row of zeros normalises to zeros (eps keeps it finite)
    assert np.all(orc.rmsnorm(np.zeros((1, 8), np.float32), np.ones(8, np.float32)) == 0)


def test_add_rmsnorm_is_add_then_rmsnorm():
    rng = np.random.default_rng(2)
    for dt in (np.float32, np.uint16):
        h = rng.standard_normal((4, 256)).astype(np.float32)
        p = rng.standard_normal((4, 256)).astype(np.float32)
        w = (1 + 0.02 * rng.standard_normal(256)).astype(np.float32)
        if dt == np.uint16:
            h, p, w = orc.f32_to_bf16(h), orc.f32_to_bf16(p), orc.f32_to_bf16(w)
        h2, y = orc.add_rmsnorm(h, p, w)
        assert np.array_equal(h2, orc.add(h, p))
        assert np.array_equal(y, orc.rmsnorm(h2, w))


def test_rope_kv_store_matches_rope_then_kv_store():
    rng = np.random.default_rng(3)
    rows, hq, hkv, hd, max_seq, seqs = 7, 6, 3, 48, 16, 2
    q = rng.uniform(-1, 1, (rows, hq, hd)).astype(np.float32)
    k = rng.uniform(-1, 1, (rows, hkv, hd)).astype(np.float32)
    v = rng.uniform(-1, 1, (rows, hkv, hd)).astype(np.float32)
    pos = np.array([0, 1, 5, 9, 15, 3, 4], np.int32)
    seq = np.array([0, 0, 1, 1, 0, 1, 0], np.int32)
    kc = np.zeros((seqs, hkv, max_seq, hd), np.float32)
    q2, kc2, vc2, bad = orc.rope_kv_store(q, k, v, pos, kc, kc, 1e4, seq_ids=seq)
    assert bad == 0
    assert np.array_equal(q2, orc.rope(q, pos, 1e4))
    want_k, _ = orc.kv_store(kc, orc.rope(k, pos, 1e4), pos, seq)
    want_v, _ = orc.kv_store(kc, v, pos, seq)
    assert np.array_equal(kc2, want_k) and np.array_equal(vc2, want_v)


def test_bad_rows_are_skipped_and_reported():
    table = np.arange(12, dtype=np.float32).reshape(4, 3)
    out, bad = orc.gather(table, np.array([1, 4, -1, 3], np.int32))
    assert bad == 0x1
    assert np.array_equal(out[0], table[1]) and np.array_equal(out[3], table[3])
    assert not out[1].any() and not out[2].any()
    c, bad = orc.kv_store(np.zeros((1, 1, 4, 2), np.float32), np.ones((2, 1, 2), np.float32),
                          np.array([4, 1], np.int32), np.array([0, 1], np.int32))
    assert bad == 0x2 | 0x4 and not c.any()


def test_torch_numpy_round_trip():
    t = torch.randn(3, 5).to(torch.bfloat16)
    assert torch.equal(from_np(to_np(t)).view(torch.int16), t.view(torch.int16))

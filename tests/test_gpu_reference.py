"""The kernels against the reference itself, on the GPU.

* The reference's unmodified test harness (tests/kernel_tests.cu), compiled
  against include/kernels.cuh and linked to libbm_layer_ops.so for the five
  layer ops (oracle/_ref/kernel_tests_dropin), passes all of its checks.
* The drop-in launch_* symbols (C++ linkage, the reference's signatures) called
  directly, and the golden RoPE vectors of the reference's reference_rope.
* The reference's own CUDA kernels (oracle/_ref/libref_kernels.so, compiled for
  sm_100a) on the same inputs, called one token per launch as
  ExecutionEngine::run_layers calls them: both implementations are graded by the
  oracle, and ours must be within 1e-5 (fp32) everywhere.
"""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest
import torch

from baremetalinferenceengine_b200 import _lib, ops
from oracle import oracle as orc
from tests.helpers import bits_equal, from_np, gen, to_np

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LEGACY = {
    "launch_rms_norm": "_Z15launch_rms_normPfS_S_ifP11CUstream_st",
    "launch_rope": "_Z11launch_ropePfS_iiiifP11CUstream_st",
    "launch_swiglu": "_Z13launch_swigluPfS_S_iP11CUstream_st",
    "launch_add": "_Z10launch_addPfS_S_iP11CUstream_st",
    "launch_kv_store": "_Z15launch_kv_storePfS_iiiiP11CUstream_st",
}
vp, ci, cf = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def legacy():
    L = _lib.load()
    fns = {}
    argtypes = {
        "launch_rms_norm": [vp, vp, vp, ci, cf, vp],
        "launch_rope": [vp, vp, ci, ci, ci, ci, cf, vp],
        "launch_swiglu": [vp, vp, vp, ci, vp],
        "launch_add": [vp, vp, vp, ci, vp],
        "launch_kv_store": [vp, vp, ci, ci, ci, ci, vp],
    }
    for name, mangled in LEGACY.items():
        fn = getattr(L, mangled)
        fn.restype = None
        fn.argtypes = argtypes[name]
        fns[name] = fn
    return fns


def ref_kernels():
    if not os.path.exists(orc.REF_KERNELS_LIB):
        pytest.fail("oracle/_ref/libref_kernels.so is missing (make -C oracle ref where the reference is present)")
    L = ctypes.CDLL(orc.REF_KERNELS_LIB)
    L.ref_rms_norm.argtypes = [vp, vp, vp, ci, cf, vp]
    L.ref_rope.argtypes = [vp, vp, ci, ci, ci, ci, cf, vp]
    L.ref_swiglu.argtypes = [vp, vp, vp, ci, vp]
    L.ref_add.argtypes = [vp, vp, vp, ci, vp]
    L.ref_kv_store.argtypes = [vp, vp, ci, ci, ci, ci, vp]
    for f in (L.ref_rms_norm, L.ref_rope, L.ref_swiglu, L.ref_add, L.ref_kv_store):
        f.restype = None
    return L


def test_reference_harness_passes_on_the_dropin(cuda):
    if not os.path.exists(orc.REF_HARNESS_DROPIN):
        pytest.fail("oracle/_ref/kernel_tests_dropin is missing (make -C oracle ref)")
    proc = subprocess.run([orc.REF_HARNESS_DROPIN], capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "0 check(s) failed" in proc.stdout
    for line in proc.stdout.splitlines():
        if line.startswith(("PASS", "FAIL")) and not line[6:].startswith(("gemm", "softmax", "attention")):
            assert line.startswith("PASS"), line
            assert float(re.search(r"worst relative error (\S+)", line).group(1)) <= 1e-5, line


def test_legacy_symbols_single_token(cuda):
    """The five drop-in symbols, called as the engine calls them (one token, fp32)."""
    f = legacy()
    g = gen(60)
    dim, hd, h, hkv, max_seq, ffn = 4096, 128, 32, 8, 64, 14336
    x, w = torch.randn(dim, generator=g), torch.rand(dim, generator=g) + 0.5
    xd, wd, outd = x.cuda(), w.cuda(), torch.empty(dim, device=cuda)
    f["launch_rms_norm"](outd.data_ptr(), xd.data_ptr(), wd.data_ptr(), dim, 1e-5, None)
    f["launch_rms_norm"](xd.data_ptr(), xd.data_ptr(), wd.data_ptr(), dim, 1e-5, None)  # in place
    want = orc.rmsnorm(x.numpy()[None], w.numpy())[0]
    assert orc.worst_error(outd.cpu().numpy(), want) <= 1e-5
    assert bits_equal(xd, outd)

    q, k = torch.randn(h * hd, generator=g), torch.randn(hkv * hd, generator=g)
    qd, kd = q.cuda(), k.cuda()
    f["launch_rope"](qd.data_ptr(), kd.data_ptr(), 4097, hd, h, hkv, 500000.0, None)
    assert orc.worst_error(qd.cpu().numpy(), orc.rope(q.numpy().reshape(1, h, hd), 4097, 5e5).ravel()) <= 1e-5
    assert orc.worst_error(kd.cpu().numpy(), orc.rope(k.numpy().reshape(1, hkv, hd), 4097, 5e5).ravel()) <= 1e-5

    gt, up = torch.randn(ffn, generator=g) * 3, torch.randn(ffn, generator=g)
    gtd, upd = gt.cuda(), up.cuda()  # kept alive: a freed temporary's block could be reused by the next copy
    act = torch.empty(ffn, device=cuda)
    f["launch_swiglu"](act.data_ptr(), gtd.data_ptr(), upd.data_ptr(), ffn, None)
    assert orc.worst_error(act.cpu().numpy(), orc.swiglu(gt.numpy(), up.numpy())) <= 1e-5

    a, b = torch.randn(dim, generator=g), torch.randn(dim, generator=g)
    ad, bd = a.cuda(), b.cuda()
    f["launch_add"](ad.data_ptr(), ad.data_ptr(), bd.data_ptr(), dim, None)
    assert bits_equal(ad, a + b)

    cache = torch.randn(hkv, max_seq, hd, generator=g)
    cd = cache.cuda()
    f["launch_kv_store"](cd.data_ptr(), kd.data_ptr(), 9, hkv, hd, max_seq, None)
    want = cache.clone()
    want[:, 9, :] = kd.cpu().view(hkv, hd)
    assert bits_equal(cd, want)


def test_golden_rope_vectors(cuda):
    """Our kernels reproduce reference_rope's own outputs (tests/golden)."""
    f = legacy()
    z = np.load(os.path.join(GOLDEN, "rope_reference.npz"))
    for n in range(int(z["count"])):
        pos, hd, heads, theta = (int(z[f"meta{n}"][0]), int(z[f"meta{n}"][1]), int(z[f"meta{n}"][2]),
                                 float(z[f"meta{n}"][3]))
        x, want = z[f"x{n}"], z[f"out{n}"]
        # the drop-in symbol (fp64 cos/sin per pair)
        qd = torch.from_numpy(x.copy()).cuda()
        f["launch_rope"](qd.data_ptr(), None, pos, hd, heads, 0, theta, None)
        assert orc.worst_error(qd.cpu().numpy(), want) <= 1e-6, n
        # the batched path with a position table
        qd = torch.from_numpy(x.copy()).cuda().view(1, heads, hd)
        ops.rope(qd, None, torch.tensor([pos], dtype=torch.int32, device=cuda),
                 table=ops.RopeTable(pos + 1, hd, theta, cuda))
        assert orc.worst_error(qd.cpu().numpy(), want) <= 1e-5, n


def _ref_per_token(fn, rows, *args):
    for r in range(rows):
        fn(*[a(r) if callable(a) else a for a in args])


def test_ours_and_the_reference_kernels_against_the_oracle(cuda):
    """Same fp32 inputs through the reference's kernels (one launch per token) and
    ours (one launch per batch). Both are graded by the oracle; the reference's
    own error is reported for context, ours must meet 1e-5."""
    R = ref_kernels()
    g = gen(70)
    rows, dim, hq, hkv, hd, ffn, max_seq, theta = 32, 4096, 32, 8, 128, 14336, 8192, 5e5
    es = 4
    report = {}

    # RMSNorm
    x, w = torch.randn(rows, dim, generator=g), 1 + 0.02 * torch.randn(dim, generator=g)
    want = orc.rmsnorm(x.numpy(), w.numpy())
    xd, wd = x.cuda(), w.cuda()
    ref_out = torch.empty_like(xd)
    _ref_per_token(R.ref_rms_norm, rows, lambda r: ref_out.data_ptr() + r * dim * es,
                   lambda r: xd.data_ptr() + r * dim * es, wd.data_ptr(), dim, 1e-5, None)
    ours = ops.rmsnorm(xd, wd)
    report["rms_norm"] = (orc.worst_error(to_np(ours), want), orc.worst_error(to_np(ref_out), want))

    # SwiGLU
    gt, up = torch.randn(rows, ffn, generator=g), torch.randn(rows, ffn, generator=g)
    want = orc.swiglu(gt.numpy(), up.numpy())
    gd, ud = gt.cuda(), up.cuda()
    ref_out = torch.empty_like(gd)
    _ref_per_token(R.ref_swiglu, rows, lambda r: ref_out.data_ptr() + r * ffn * es,
                   lambda r: gd.data_ptr() + r * ffn * es, lambda r: ud.data_ptr() + r * ffn * es, ffn, None)
    ours = ops.swiglu(gd, ud)
    report["swiglu"] = (orc.worst_error(to_np(ours), want), orc.worst_error(to_np(ref_out), want))

    # RoPE + KV store (reference: launch_rope then launch_kv_store x2 per token, one sequence)
    q, k, v = (torch.randn(rows, n, hd, generator=g) for n in (hq, hkv, hkv))
    pos = torch.randint(0, max_seq, (rows,), generator=g, dtype=torch.int32)
    pos = torch.unique(pos)[:rows]
    rows_r = pos.numel()
    q, k, v = q[:rows_r], k[:rows_r], v[:rows_r]
    cache0 = torch.zeros(1, hkv, max_seq, hd)
    want_q, want_kc, want_vc, _ = orc.rope_kv_store(q.numpy(), k.numpy(), v.numpy(), pos.numpy(), cache0.numpy(),
                                                    cache0.numpy(), theta)
    qr, kr, vr = q.cuda(), k.cuda(), v.cuda()
    kcr, vcr = cache0.cuda(), cache0.cuda()
    for r in range(rows_r):
        p = int(pos[r])
        R.ref_rope(qr[r].data_ptr(), kr[r].data_ptr(), p, hd, hq, hkv, theta, None)
        R.ref_kv_store(kcr.data_ptr(), kr[r].data_ptr(), p, hkv, hd, max_seq, None)
        R.ref_kv_store(vcr.data_ptr(), vr[r].data_ptr(), p, hkv, hd, max_seq, None)
    qo, kco, vco = q.cuda(), cache0.cuda(), cache0.cuda()
    ops.rope_kv_store(qo, k.cuda(), v.cuda(), pos.cuda(), kco, vco, table=ops.RopeTable(max_seq, hd, theta, cuda),
                      theta=theta)
    report["rope_q"] = (orc.worst_error(to_np(qo), want_q), orc.worst_error(to_np(qr), want_q))
    report["rope_k_cache"] = (orc.worst_error(to_np(kco), want_kc), orc.worst_error(to_np(kcr), want_kc))
    assert bits_equal(vco, vcr) and bits_equal(vco, from_np(want_vc))

    # add (in place, as the engine's residual add)
    a, b = torch.randn(rows, dim, generator=g), torch.randn(rows, dim, generator=g)
    ar, ao, bd = a.cuda(), a.cuda(), b.cuda()
    R.ref_add(ar.data_ptr(), ar.data_ptr(), bd.data_ptr(), rows * dim, None)
    ops.add(ao, b.cuda(), out=ao)
    assert bits_equal(ao, ar)

    print("worst error vs oracle (ours, reference kernels):", report)
    for name, (ours_err, ref_err) in report.items():
        assert ours_err <= 1e-5, (name, ours_err, ref_err)


def test_reference_engine_runs_on_the_dropin(cuda, tmp_path):
    """The reference's ExecutionEngine and its logits test (tests/logits_test.cu),
    unmodified, built against this library for the five layer ops, reproduce the
    logits of the same engine on the reference's own kernels: every position within
    the test's 0.01 limit, the same next token everywhere, and the same logits after
    a reset with the whole sequence in one call. The model is a seeded synthetic
    export (no checkpoint is available); golden logits come from
    oracle/_ref/engine_golden_ref (the reference's engine and kernels)."""
    from tests.engine_export import write_export

    for exe in ("engine_golden_ref", "logits_test_dropin"):
        if not os.path.exists(os.path.join(orc.REF_DIR, exe)):
            pytest.fail(f"oracle/_ref/{exe} is missing (make -C oracle ref)")
    cfg = write_export(str(tmp_path), seed=11)
    tokens = [int(t) for t in np.random.default_rng(12).integers(0, cfg["vocab"], 40)]
    gold = subprocess.run([os.path.join(orc.REF_DIR, "engine_golden_ref"), str(tmp_path)] + [str(t) for t in tokens],
                          capture_output=True, text=True, timeout=600)
    assert gold.returncode == 0, gold.stdout[-2000:] + gold.stderr[-2000:]
    run = subprocess.run([os.path.join(orc.REF_DIR, "logits_test_dropin"), str(tmp_path)], capture_output=True,
                         text=True, timeout=600)
    print(run.stdout[-1500:])
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-2000:]
    assert "0 check(s) failed" in run.stdout

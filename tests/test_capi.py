"""CPU-side checks of the C ABI library (no kernel launches).

* libbm_layer_ops.so loads and exports every entry point include/bm_layer_ops.h
  declares, and the five C++ launch_* symbols of include/kernels.cuh with the
  reference's exact mangled signatures (include/kernels.cuh:9,15,29,32,36).
* Host-side argument checks reject bad input before anything reaches CUDA, and
  zero-size calls return BM_OK without a launch.
* The oracle's reference-built files and the drop-in harness link as expected.
"""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from baremetalinferenceengine_b200 import _lib, build
from tests.helpers import reference_dir

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "bm_layer_ops.h")

# The reference's mangled launch symbols (g++ Itanium ABI for include/kernels.cuh).
LEGACY = {
    "launch_rms_norm": "_Z15launch_rms_normPfS_S_ifP11CUstream_st",
    "launch_rope": "_Z11launch_ropePfS_iiiifP11CUstream_st",
    "launch_swiglu": "_Z13launch_swigluPfS_S_iP11CUstream_st",
    "launch_add": "_Z10launch_addPfS_S_iP11CUstream_st",
    "launch_kv_store": "_Z15launch_kv_storePfS_iiiiP11CUstream_st",
    "launch_attention": "_Z16launch_attentionPfS_S_S_S_iiiiP11CUstream_st",
    "launch_gemm": "_Z11launch_gemmPfS_S_iiiP11CUstream_st",
    "launch_softmax": "_Z14launch_softmaxPfiP11CUstream_st",
    "launch_softmax_batch": "_Z20launch_softmax_batchPfiiiP11CUstream_st",
}


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(bm_\w+)\(", text, re.M)))


def test_header_declares_every_binding():
    names = declared_symbols()
    assert len(names) >= 14
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_library_exports_the_reference_launch_symbols(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.lib_path()], capture_output=True, text=True).stdout
    for mangled in LEGACY.values():
        assert re.search(rf"\sT\s{mangled}$", out, re.M), mangled


def test_legacy_symbols_match_the_reference_header():
    """Mangle the reference's own declarations with g++ and compare."""
    ref = reference_dir()
    if ref is None:
        pytest.skip("the reference's sources are not present")
    src = '#include "kernels.cuh"\n' + "\n".join(
        f"void* p_{n} = (void*)&{n};" for n in LEGACY)
    with tempfile.TemporaryDirectory() as tmp:
        obj = os.path.join(tmp, "probe.o")
        proc = subprocess.run(["g++", "-x", "c++", "-c", "-o", obj, f"-I{ref}/include",
                               "-I/usr/local/cuda/include", "-"], input=src.encode(), capture_output=True)
        assert proc.returncode == 0, proc.stderr.decode()
        syms = subprocess.run(["nm", "-u", obj], capture_output=True, text=True).stdout
    for mangled in LEGACY.values():
        assert mangled in syms


def test_abi_version_and_status_strings(lib):
    assert lib.bm_abi_version() == 1
    for code, name in [(0, b"BM_OK"), (1, b"BM_ERR_INVALID_ARGUMENT"), (2, b"BM_ERR_CUDA"), (3, b"BM_ERR_DEVICE")]:
        assert lib.bm_status_string(code) == name
    assert lib.bm_status_string(99) == b"BM_ERR_UNKNOWN"


FAKE = 0x100000  # never dereferenced: every call below fails or returns before any CUDA call
PTRS3 = (ctypes.c_void_p * 3)(FAKE, FAKE, FAKE)  # host arrays of (fake) device pointers
WIDTHS3 = (ctypes.c_int32 * 3)(8, 8, 8)
WIDTHS_BAD = (ctypes.c_int32 * 3)(8, -1, 8)
WIDTHS_UNEQUAL = (ctypes.c_int32 * 3)(8, 16, 8)


def rope_attn(L, table=FAKE, table_len=8, positions=FAKE, hd=64, batch=1):
    """bm_rope_kv_decode_attention with fake pointers: 2 heads, max_seq 8, fp32."""
    return L.bm_rope_kv_decode_attention(FAKE, FAKE, FAKE, FAKE, positions, table, table_len, None, FAKE, FAKE,
                                         FAKE, 8, batch, 2, 2, hd, 8, 1, 0.0, None, 0, 0, None, None)


def norm_gemm(L, c=PTRS3, h=FAKE, d=None, res=None, normed=FAKE * 8, widths=WIDTHS3, count=3, swiglu=0, m=4, k=8,
              dtype=0):
    """bm_rmsnorm_gemm with fake pointers."""
    return L.bm_rmsnorm_gemm(c, h, d, FAKE, 1e-5, res, normed, PTRS3, widths, count, swiglu, m, k, dtype, None, None)


@pytest.mark.parametrize("call", [
    lambda L: L.bm_rmsnorm(FAKE, FAKE, FAKE, 4, 64, 1e-5, 64, 64, 7, None),          # bad dtype
    lambda L: L.bm_rmsnorm(FAKE, FAKE, FAKE, -1, 64, 1e-5, 64, 64, 0, None),         # negative rows
    lambda L: L.bm_rmsnorm(FAKE, FAKE, FAKE, 4, 64, 1e-5, 32, 64, 0, None),          # stride < dim
    lambda L: L.bm_rmsnorm(None, FAKE, FAKE, 4, 64, 1e-5, 64, 64, 0, None),          # NULL out
    lambda L: L.bm_rmsnorm(FAKE, FAKE, FAKE, 4, 64, -1.0, 64, 64, 0, None),          # eps < 0
    lambda L: L.bm_rmsnorm(FAKE + 64, FAKE, FAKE, 4, 64, 1e-5, 64, 64, 0, None),     # partial overlap
    lambda L: L.bm_add_rmsnorm(FAKE, FAKE, FAKE, FAKE, 4, 64, 1e-5, 0, None),        # out overlaps residual
    lambda L: L.bm_add_rmsnorm(FAKE, None, FAKE, FAKE * 4, 4, 64, 1e-5, 0, None),    # NULL delta
    lambda L: L.bm_swiglu(FAKE, FAKE, FAKE, -5, 0, None),                            # negative n
    lambda L: L.bm_swiglu(FAKE + 4, FAKE, FAKE * 4, 64, 0, None),                    # partial overlap
    lambda L: L.bm_add(FAKE, None, FAKE, 8, 1, None),                                # NULL input
    lambda L: L.bm_embed_gather(FAKE, FAKE, FAKE, 4, 64, 10, 32, 0, None, None),     # pitch < dim
    lambda L: L.bm_embed_gather(FAKE, FAKE, FAKE, 4, 64, 1 << 40, 64, 0, None, None),  # vocab > int32
    lambda L: L.bm_rope(FAKE, FAKE, None, 0, None, 0, 1e4, 1, 2, 2, 7, 0, None, None),  # odd head_dim
    lambda L: L.bm_rope(FAKE, FAKE, None, 0, None, 0, 0.0, 1, 2, 2, 8, 0, None, None),  # theta 0, no table
    lambda L: L.bm_rope(FAKE, FAKE, None, 0, FAKE, 0, 1e4, 1, 2, 2, 8, 0, None, None),  # table_len 0
    lambda L: L.bm_rope(FAKE, FAKE, None, 0, FAKE + 4, 8, 1e4, 1, 2, 2, 8, 0, None, None),  # table misaligned
    lambda L: L.bm_rope(FAKE, FAKE, None, 0, None, 0, 1e4, 1, 2, 2, 2048, 0, None, None),  # head_dim > 1024
    lambda L: L.bm_rope_kv_store(FAKE, FAKE, FAKE, None, 7, None, FAKE, FAKE, None, 0, 1e4, 2, 2, 1, 8, 8, 1, 0,
                                 None, None),                                          # pos0 + rows > max_seq
    lambda L: L.bm_rope_kv_store(FAKE, FAKE, None, FAKE, 0, None, FAKE, FAKE, None, 0, 1e4, 2, 2, 1, 8, 8, 1, 0,
                                 None, None),                                          # NULL v
    lambda L: L.bm_rope_kv_store(FAKE, FAKE, FAKE, FAKE, 0, None, FAKE, FAKE, None, 0, 1e4, 2, 2, 1, 8, 8, 0, 0,
                                 None, None),                                          # num_seqs 0
    lambda L: L.bm_kv_store(FAKE, FAKE, None, -1, None, 1, 2, 8, 8, 1, 0, None, None),  # negative pos0
    lambda L: L.bm_kv_store(FAKE, FAKE, None, 0, None, 1, 2, 8, 0, 1, 0, None, None),   # max_seq 0
    lambda L: L.bm_rope_table_fill(FAKE, 8, 7, 1e4, None),                            # odd head_dim
    lambda L: L.bm_rope_table_fill(FAKE, 0, 8, 1e4, None),                            # max_pos 0
    lambda L: L.bm_rope_table_create(8, 8, -1.0, ctypes.byref(ctypes.c_void_p())),     # theta < 0
    lambda L: L.bm_kv_cache_create(0, 1, 1, 8, 8, 8, 0, ctypes.byref(ctypes.c_void_p())),  # no layers
    lambda L: L.bm_kv_cache_create(1, 1, 1, 8, 8, 0, 0, ctypes.byref(ctypes.c_void_p())),  # max_tokens 0
    lambda L: L.bm_kv_cache_create(1, 1, 1, 8, 8, 8, 5, ctypes.byref(ctypes.c_void_p())),  # bad dtype
    lambda L: L.bm_kv_cache_create(1, 1, 1, 8, 8, 8, 0, None),                        # NULL out
    lambda L: L.bm_kv_cache_append(None, None, 0, ctypes.byref(ctypes.c_void_p()), ctypes.byref(ctypes.c_void_p()),
                                   None),                                               # NULL cache
    lambda L: L.bm_kv_cache_layer(None, 0, ctypes.byref(ctypes.c_void_p()), ctypes.byref(ctypes.c_void_p())),
    lambda L: L.bm_kv_cache_seq_len(None, 0, ctypes.byref(ctypes.c_int32())),
    lambda L: L.bm_kv_cache_reset(None, 0),
    lambda L: L.bm_gemm(FAKE, FAKE, FAKE, 3, 5, 7, 1, None, None),                    # N, K not multiples of 8
    lambda L: L.bm_gemm(FAKE, FAKE, FAKE, 4, 64, 60, 1, None, None),                  # K not a multiple of 8
    lambda L: L.bm_gemm(FAKE, FAKE, FAKE, -1, 64, 64, 1, None, None),                 # negative rows
    lambda L: L.bm_gemm(FAKE, FAKE + 2, FAKE, 4, 64, 64, 1, None, None),              # misaligned operand
    lambda L: L.bm_gemm(FAKE, None, FAKE, 4, 64, 64, 1, None, None),                  # NULL operand
    lambda L: L.bm_gemm_swiglu(FAKE, FAKE, FAKE, FAKE, -4, 64, 64, 0, None, None),   # fp32: negative rows
    lambda L: L.bm_gemm_swiglu(FAKE, FAKE, None, FAKE, 4, 64, 64, 0, None, None),    # fp32: NULL w_gate
    lambda L: L.bm_gemm_swiglu(FAKE, FAKE, FAKE, FAKE, 4, 64, 60, 1, None, None),    # hidden % 8
    lambda L: L.bm_gemm_swiglu(FAKE, FAKE, FAKE, None, 4, 64, 64, 1, None, None),    # NULL w_up
    lambda L: L.bm_gemm(FAKE, None, FAKE, 4, 5, 7, 0, None, None),                    # fp32: NULL operand
    lambda L: L.bm_gemm(FAKE, FAKE, FAKE, -1, 5, 7, 0, None, None),                   # fp32: negative rows
    lambda L: L.bm_softmax(FAKE, 8, 2, 4, 0, None),                                   # stride < size
    lambda L: L.bm_softmax(FAKE, -1, 1, 8, 0, None),                                  # negative size
    lambda L: L.bm_softmax(None, 8, 1, 8, 0, None),                                   # NULL x
    lambda L: L.bm_softmax(FAKE, 8, 1, 8, 9, None),                                   # bad dtype
    lambda L: L.bm_gemm_shared_a(None, FAKE, None, None, 1, 4, 8, 0, None, None),    # NULL arrays
    lambda L: L.bm_gemm_shared_a(PTRS3, FAKE, PTRS3, WIDTHS_BAD, 3, 4, 8, 0, None, None),  # negative width
    lambda L: L.bm_gemm_shared_a(PTRS3, FAKE, PTRS3, WIDTHS3, 0, 4, 8, 0, None, None),     # count 0
    lambda L: L.bm_gemm_shared_a(PTRS3, FAKE, PTRS3, WIDTHS3, 4, 4, 8, 0, None, None),     # count 4
    lambda L: L.bm_gemm_shared_a(PTRS3, None, PTRS3, WIDTHS3, 3, 4, 8, 0, None, None),     # NULL a
    lambda L: L.bm_gemm_shared_a(PTRS3, FAKE, PTRS3, WIDTHS3, 3, 4, 8, 9, None, None),     # bad dtype
    lambda L: norm_gemm(L, c=None),                                                   # NULL output array
    lambda L: norm_gemm(L, count=0),                                                  # count 0
    lambda L: norm_gemm(L, swiglu=1),                                                 # swiglu takes 2 weights
    lambda L: norm_gemm(L, count=2, swiglu=1, widths=WIDTHS_UNEQUAL),                 # gate / up widths differ
    lambda L: norm_gemm(L, k=0),                                                      # empty rows: no norm
    lambda L: norm_gemm(L, normed=None),                                              # NULL scratch
    lambda L: norm_gemm(L, d=FAKE * 4, res=FAKE),                                     # residual_out over h
    lambda L: norm_gemm(L, d=FAKE * 4, res=FAKE * 4 + 16),                            # residual_out over d
    lambda L: norm_gemm(L, dtype=9),                                                  # bad dtype
    lambda L: rope_attn(L, table=None),                                               # the table is required
    lambda L: rope_attn(L, table_len=0),                                              # empty table
    lambda L: rope_attn(L, table=FAKE + 4),                                           # table misaligned
    lambda L: rope_attn(L, positions=None),                                           # NULL positions
    lambda L: rope_attn(L, hd=6),                                                     # rows not 16-byte vectors
    lambda L: L.bm_selftest_bounded_wait(1000, FAKE, FAKE, None),                     # limit below 1 ms
    lambda L: L.bm_selftest_bounded_wait(10**10, FAKE, FAKE, None),                   # limit above 2 s
    lambda L: L.bm_selftest_bounded_wait(50 * 10**6, None, FAKE, None),               # NULL status
])
def test_host_checks_reject_before_any_launch(lib, call):
    assert call(lib) == _lib.BM_ERR_INVALID_ARGUMENT
    assert lib.bm_last_error_message()  # a reason is recorded


@pytest.mark.parametrize("call", [
    lambda L: L.bm_rmsnorm(FAKE, FAKE, FAKE, 0, 64, 1e-5, 64, 64, 0, None),
    lambda L: L.bm_add_rmsnorm(FAKE, FAKE, FAKE, FAKE * 4, 4, 0, 1e-5, 1, None),
    lambda L: L.bm_swiglu(FAKE, FAKE, FAKE, 0, 1, None),
    lambda L: L.bm_add(FAKE, FAKE, FAKE, 0, 0, None),
    lambda L: L.bm_embed_gather(FAKE, FAKE, FAKE, 0, 64, 10, 64, 0, None, None),
    lambda L: L.bm_rope(FAKE, FAKE, None, 0, None, 0, 1e4, 0, 2, 2, 8, 0, None, None),
    lambda L: L.bm_rope_kv_store(FAKE, FAKE, FAKE, None, 0, None, FAKE, FAKE, None, 0, 1e4, 0, 2, 1, 8, 8, 1, 0,
                                 None, None),
    lambda L: L.bm_kv_store(FAKE, FAKE, None, 0, None, 0, 2, 8, 8, 1, 0, None, None),
    lambda L: L.bm_rope_table_destroy(None),
    lambda L: L.bm_kv_cache_destroy(None),
    lambda L: L.bm_gemm(FAKE, FAKE, FAKE, 0, 64, 64, 1, None, None),
    lambda L: L.bm_gemm_swiglu(FAKE, FAKE, FAKE, FAKE, 0, 64, 64, 1, None, None),
    lambda L: L.bm_gemm(FAKE, FAKE, FAKE, 0, 5, 7, 0, None, None),
    lambda L: L.bm_softmax(FAKE, 0, 4, 8, 0, None),
    lambda L: L.bm_softmax(FAKE, 8, 0, 8, 0, None),
    lambda L: norm_gemm(L, m=0),
    lambda L: rope_attn(L, batch=0),
])
def test_empty_calls_are_no_ops(lib, call):
    assert call(lib) == _lib.BM_OK


def test_status_read_rejects_null(lib):
    assert lib.bm_status_read(None, None, None) == _lib.BM_ERR_INVALID_ARGUMENT


def test_ops_layer_rejects_unsupported_dtypes_without_cuda():
    import torch

    from baremetalinferenceengine_b200 import ops

    with pytest.raises(_lib.BMError):
        ops.bm_dtype(torch.zeros(1, dtype=torch.float16))
    with pytest.raises(_lib.BMError):
        ops.swiglu(torch.zeros(4), torch.zeros(4))  # CPU tensors: not a CUDA device


def test_dropin_harness_links_against_this_library():
    from oracle import oracle as orc

    if not os.path.exists(orc.REF_HARNESS_DROPIN):
        pytest.skip("oracle/_ref/kernel_tests_dropin not built")
    out = subprocess.run(["ldd", orc.REF_HARNESS_DROPIN], capture_output=True, text=True).stdout
    assert "libbm_layer_ops.so" in out
    und = subprocess.run(["nm", "-u", orc.REF_HARNESS_DROPIN], capture_output=True, text=True).stdout
    for mangled in LEGACY.values():
        assert mangled in und  # resolved from libbm_layer_ops.so, not the reference's kernels


def test_layer_step_struct_layout_matches_the_header():
    """The ctypes mirror of bm_layer_step_t has the C struct's size and field
    offsets (gcc compiles the header and prints them)."""
    fields = [name for name, _ in _lib.LayerStepC._fields_]
    src = '#include <stddef.h>\n#include <stdio.h>\n#include "bm_layer_ops.h"\nint main(void) {\n'
    src += '  printf("%zu\\n", sizeof(bm_layer_step_t));\n'
    for f in fields:
        src += f'  printf("%zu\\n", offsetof(bm_layer_step_t, {f}));\n'
    src += "  return 0;\n}\n"
    with tempfile.TemporaryDirectory() as tmp:
        c, exe = os.path.join(tmp, "layout.c"), os.path.join(tmp, "layout")
        with open(c, "w") as fh:
            fh.write(src)
        inc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
        proc = subprocess.run(["gcc", "-std=c11", "-I", inc, "-I/usr/local/cuda/include", "-o", exe, c],
                              capture_output=True, text=True)
        assert proc.returncode == 0, proc.stderr
        out = [int(x) for x in subprocess.run([exe], capture_output=True, text=True).stdout.split()]
    assert out[0] == ctypes.sizeof(_lib.LayerStepC)
    for f, off in zip(fields, out[1:]):
        assert getattr(_lib.LayerStepC, f).offset == off, f

"""TEST INFRASTRUCTURE: numpy/ctypes front end of the CPU oracle (bm_oracle.c).

The oracle restates the reference's double-precision check loops
(tests/kernel_tests.cu:75-79, 122, 175-187, 206, 223-226 and the row copy of
src/execution_engine.cu:98-99); every function here cites the C routine it
calls. Arrays are numpy: fp32 as float32, bf16 as uint16 bit patterns.

``ref_*`` functions call the reference's own compiled CPU code
(oracle/_ref/libref_cpu.so, built from the reference's unmodified
tests/kernel_tests.cu by oracle/Makefile) and exist only where that build is
present.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_CPU_LIB = os.path.join(REF_DIR, "libref_cpu.so")
REF_KERNELS_LIB = os.path.join(REF_DIR, "libref_kernels.so")
REF_HARNESS_CPU = os.path.join(REF_DIR, "ref_kernel_tests_on_oracle")
REF_HARNESS_DROPIN = os.path.join(REF_DIR, "kernel_tests_dropin")

F32, BF16 = 0, 1

_lib = None
_ref = None

vp, i64, i32, dbl, cint = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_double, ctypes.c_int


class OracleStep(ctypes.Structure):
    """Mirror of ``OracleStep`` in bm_oracle.c (one layer step's sizes and buffers)."""

    _fields_ = [
        ("rows", i64), ("dim", i64), ("vocab", i64), ("ffn", i64),
        ("hq", i32), ("hkv", i32), ("hd", i32), ("max_seq", i32), ("num_seqs", i32), ("table_len", i32),
        ("eps", dbl), ("theta", dbl), ("dtype", i32),
        ("ids", vp), ("embed", vp), ("hidden", vp), ("attn_out", vp), ("w_attn", vp), ("normed", vp),
        ("q", vp), ("k", vp), ("v", vp), ("positions", vp), ("seq_ids", vp), ("k_cache", vp), ("v_cache", vp),
        ("ffn_out", vp), ("w_ffn", vp), ("gate", vp), ("up", vp), ("act", vp),
        ("ops", i32),
    ]


def build() -> str:
    """Compiles liboracle.so (gcc) when missing or older than bm_oracle.c."""
    src = os.path.join(HERE, "bm_oracle.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        sig = {
            "oracle_rmsnorm": (None, [vp, vp, vp, i64, i64, dbl, i64, i64, cint]),
            "oracle_add": (None, [vp, vp, vp, i64, cint]),
            "oracle_add_rmsnorm": (None, [vp, vp, vp, vp, i64, i64, dbl, cint]),
            "oracle_swiglu": (None, [vp, vp, vp, i64, cint]),
            "oracle_rope": (None, [vp, vp, i32, i64, cint, cint, dbl, cint]),
            "oracle_kv_store": (i32, [vp, vp, vp, i32, vp, i64, cint, cint, cint, cint, cint]),
            "oracle_rope_kv_store": (i32, [vp, vp, vp, vp, i32, vp, vp, vp, i32, dbl, i64, cint, cint, cint, cint,
                                           cint, cint]),
            "oracle_rope_table": (None, [vp, i32, cint, dbl]),
            "oracle_gather": (i32, [vp, vp, vp, i64, i64, i64, i64, cint]),
            "oracle_decode_attention": (i32, [vp, vp, vp, vp, vp, vp, i64, cint, cint, cint, cint, cint, cint]),
            "oracle_gemm": (None, [vp, vp, vp, i64, i64, i64, cint, cint]),
            "oracle_gemm_swiglu": (None, [vp, vp, vp, vp, i64, i64, i64, cint, cint]),
            "oracle_softmax": (None, [vp, i64, i64, i64, cint]),
            "oracle_layer_step": (i32, [ctypes.POINTER(OracleStep), i64, i64]),
            "oracle_layer_step_mt": (i32, [ctypes.POINTER(OracleStep), i64, i64, cint]),
            "oracle_f32_to_bf16": (ctypes.c_uint16, [ctypes.c_float]),
            "oracle_f64_to_bf16": (ctypes.c_uint16, [dbl]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def _dt(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.uint16:
        return BF16
    raise TypeError(f"oracle arrays are float32 or uint16 (bf16 bits), got {a.dtype}")


def _c(a):
    return None if a is None else np.ascontiguousarray(a)


# ---------------------------------------------------------------- bf16 helpers

def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round-to-nearest-even (oracle_f32_to_bf16 vectorised)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((b[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def to_f64(a: np.ndarray) -> np.ndarray:
    return bf16_to_f32(a).astype(np.float64) if a.dtype == np.uint16 else a.astype(np.float64)


# ---------------------------------------------------------------- the ops

def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """oracle_rmsnorm (tests/kernel_tests.cu:75-79) over the rows of x [rows, dim]."""
    # Every array a C call reads is bound to a name first: a temporary copy's
    # memory could be freed before the call runs.
    x, w = _c(x), _c(w)
    out = np.empty_like(x)
    dim = x.shape[-1]
    rows = x.size // dim if dim else 0
    lib().oracle_rmsnorm(_p(out), _p(x), _p(w), rows, dim, eps, dim, dim, _dt(x))
    return out


def add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """oracle_add (tests/kernel_tests.cu:206): fp32 sum, stored in the dtype."""
    a, b = _c(a), _c(b)
    out = np.empty_like(a)
    lib().oracle_add(_p(out), _p(a), _p(b), a.size, _dt(a))
    return out


def add_rmsnorm(h: np.ndarray, p: np.ndarray, w: np.ndarray, eps: float = 1e-5):
    """Returns (h + p, rmsnorm(h + p) * w): oracle_add_rmsnorm."""
    h2 = np.array(h, copy=True, order="C")
    p, w = _c(p), _c(w)
    y = np.empty_like(h2)
    dim = h2.shape[-1]
    lib().oracle_add_rmsnorm(_p(h2), _p(p), _p(w), _p(y), h2.size // dim, dim, eps, _dt(h2))
    return h2, y


def swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """oracle_swiglu (tests/kernel_tests.cu:122): g / (1 + exp(-g)) * u in double."""
    g, u = _c(g), _c(u)
    out = np.empty_like(g)
    lib().oracle_swiglu(_p(out), _p(g), _p(u), g.size, _dt(g))
    return out


def rope(x: np.ndarray, positions, theta: float) -> np.ndarray:
    """oracle_rope (reference_rope, tests/kernel_tests.cu:175-187) on x [rows, heads, hd];
    positions: int32 array or int pos0."""
    out = np.array(x, copy=True, order="C")
    rows, heads, hd = out.shape
    pos_arr = None if isinstance(positions, (int, np.integer)) else np.ascontiguousarray(positions, np.int32)
    pos0 = int(positions) if pos_arr is None else 0
    lib().oracle_rope(_p(out), _p(pos_arr), pos0, rows, heads, hd, theta, _dt(out))
    return out


def kv_store(cache: np.ndarray, src: np.ndarray, positions, seq_ids=None):
    """oracle_kv_store (tests/kernel_tests.cu:223-226) into a copy of cache
    [num_seqs, H, max_seq, hd]; returns (cache, bad_bits)."""
    c = np.array(cache, copy=True, order="C")
    rows, heads, hd = src.shape
    pos_arr = None if isinstance(positions, (int, np.integer)) else np.ascontiguousarray(positions, np.int32)
    pos0 = int(positions) if pos_arr is None else 0
    seq = None if seq_ids is None else np.ascontiguousarray(seq_ids, np.int32)
    src = _c(src)
    bad = lib().oracle_kv_store(_p(c), _p(src), _p(pos_arr), pos0, _p(seq), rows, heads, hd, c.shape[2],
                                c.shape[0], _dt(c))
    return c, bad


def rope_kv_store(q, k, v, positions, k_cache, v_cache, theta, seq_ids=None, table_len=0):
    """oracle_rope_kv_store: returns (q_rotated, k_cache, v_cache, bad_bits) on copies."""
    q2 = np.array(q, copy=True, order="C")
    kc = np.array(k_cache, copy=True, order="C")
    vc = np.array(v_cache, copy=True, order="C")
    rows, hq, hd = q2.shape
    hkv = k.shape[1]
    pos_arr = None if isinstance(positions, (int, np.integer)) else np.ascontiguousarray(positions, np.int32)
    pos0 = int(positions) if pos_arr is None else 0
    seq = None if seq_ids is None else np.ascontiguousarray(seq_ids, np.int32)
    k, v = _c(k), _c(v)
    bad = lib().oracle_rope_kv_store(_p(q2), _p(k), _p(v), _p(pos_arr), pos0, _p(seq), _p(kc), _p(vc),
                                     table_len, theta, rows, hq, hkv, hd, kc.shape[2], kc.shape[0], _dt(q2))
    return q2, kc, vc, bad


def rope_table(max_pos: int, hd: int, theta: float) -> np.ndarray:
    """oracle_rope_table: [max_pos, hd/2, 2] float32 (cos, sin)."""
    t = np.empty((max_pos, hd // 2, 2), np.float32)
    lib().oracle_rope_table(_p(t), max_pos, hd, theta)
    return t


def gather(table: np.ndarray, ids: np.ndarray, out: np.ndarray | None = None):
    """oracle_gather: row copy (src/execution_engine.cu:98-99); returns (out, bad_bits)."""
    table = _c(table)
    ids = np.ascontiguousarray(ids, np.int32)
    vocab, dim = table.shape
    if out is None:
        out = np.zeros((ids.size, dim), table.dtype)
    bad = lib().oracle_gather(_p(out), _p(table), _p(ids), ids.size, dim, vocab, dim, _dt(table))
    return out, bad


def gemm(a: np.ndarray, b: np.ndarray, threads: int = 1) -> np.ndarray:
    """oracle_gemm (reference_gemm, tests/kernel_tests.cu:49-59): a [m, k] @ b [k, n]."""
    a, b = _c(a), _c(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), a.dtype)
    lib().oracle_gemm(_p(c), _p(a), _p(b), m, n, k, _dt(a), threads)
    return c


def gemm_swiglu(x: np.ndarray, w_gate: np.ndarray, w_up: np.ndarray, threads: int = 1) -> np.ndarray:
    """oracle_gemm_swiglu: silu(x @ w_gate) * (x @ w_up) in double, rounded once
    (src/execution_engine.cu:122-124); x [rows, dim], weights [dim, hidden]."""
    x, w_gate, w_up = _c(x), _c(w_gate), _c(w_up)
    rows, dim = x.shape
    hidden = w_gate.shape[1]
    out = np.empty((rows, hidden), x.dtype)
    lib().oracle_gemm_swiglu(_p(out), _p(x), _p(w_gate), _p(w_up), rows, dim, hidden, _dt(x), threads)
    return out


def softmax(x: np.ndarray, size: int | None = None, num_vectors: int = 1, stride: int | None = None) -> np.ndarray:
    """oracle_softmax (tests/kernel_tests.cu:105-160) on a copy of the flat array x:
    num_vectors vectors of `size` elements, `stride` apart (gaps untouched)."""
    out = np.array(x, copy=True, order="C").ravel()
    size = out.size if size is None else size
    stride = size if stride is None else stride
    lib().oracle_softmax(_p(out), size, num_vectors, stride, _dt(out))
    return out.reshape(np.shape(x))


def layer_step(step: OracleStep, r0: int, r1: int, threads: int = 1) -> int:
    """oracle_layer_step(_mt) over rows [r0, r1): the timed CPU baseline."""
    if threads > 1:
        return lib().oracle_layer_step_mt(ctypes.byref(step), r0, r1, threads)
    return lib().oracle_layer_step(ctypes.byref(step), r0, r1)


# ---------------------------------------------------------------- tolerance

def worst_error(got: np.ndarray, want: np.ndarray) -> float:
    """The reference's error metric |got - want| / (1 + |want|), NaN counting as a
    failure (tests/kernel_tests.cu:36-47); inputs in any dtype (bf16 as uint16)."""
    g, w = to_f64(np.asarray(got)).ravel(), to_f64(np.asarray(want)).ravel()
    if g.size == 0:
        return 0.0
    err = np.abs(g - w) / (1.0 + np.abs(w))
    if np.isnan(err).any():
        return float("inf")
    return float(err.max())


# ---------------------------------------------------------------- reference CPU code

def ref_available() -> bool:
    return os.path.exists(REF_CPU_LIB)


def ref_lib() -> ctypes.CDLL:
    """oracle/_ref/libref_cpu.so: the reference's own tests/kernel_tests.cu."""
    global _ref
    if _ref is None:
        L = ctypes.CDLL(REF_CPU_LIB)
        L.ref_reference_rope.restype = None
        L.ref_reference_rope.argtypes = [vp, vp, cint, cint, cint, dbl]
        L.ref_reference_gemm.restype = None
        L.ref_reference_gemm.argtypes = [vp, vp, vp, cint, cint, cint]
        L.ref_kernel_tests_main.restype = cint
        L.ref_kernel_tests_main.argtypes = []
        _ref = L
    return _ref


def ref_reference_rope(x: np.ndarray, seq_pos: int, theta: float) -> np.ndarray:
    """reference_rope (tests/kernel_tests.cu:175-187) itself, on x [heads, hd] float32."""
    x = np.ascontiguousarray(x, np.float32)
    heads, hd = x.shape
    out = np.empty_like(x)
    ref_lib().ref_reference_rope(_p(out), _p(x), seq_pos, hd, heads, theta)
    return out


def ref_reference_gemm(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """reference_gemm (tests/kernel_tests.cu:49-59) itself: a [m, k] @ b [k, n], float32."""
    a, b = np.ascontiguousarray(a, np.float32), np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    ref_lib().ref_reference_gemm(_p(c), _p(a), _p(b), m, n, k)
    return c

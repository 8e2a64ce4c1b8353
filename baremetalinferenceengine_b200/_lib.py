"""ctypes binding of ``libbm_layer_ops.so`` (the C ABI in ``include/bm_layer_ops.h``).

Loading fails loudly when the library has not been built: there is no CPU or
PyTorch fallback for any op.
"""
from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

c_int, c_int32, c_int64, c_float, c_double = (ctypes.c_int, ctypes.c_int32, ctypes.c_int64,
                                              ctypes.c_float, ctypes.c_double)
c_void_p, c_char_p = ctypes.c_void_p, ctypes.c_char_p
P_INT32 = ctypes.POINTER(ctypes.c_int32)

BM_OK = 0
BM_ERR_INVALID_ARGUMENT = 1
BM_ERR_CUDA = 2
BM_ERR_DEVICE = 3

BM_F32 = 0
BM_BF16 = 1

BM_DEVERR_BAD_ID = 0x1
BM_DEVERR_BAD_POSITION = 0x2
BM_DEVERR_BAD_SEQUENCE = 0x4
BM_DEVERR_TIMEOUT = 0x8

class LayerStepC(ctypes.Structure):
    """Mirror of bm_layer_step_t (include/bm_layer_ops.h): one layer step's sizes
    and device buffers."""

    _fields_ = [
        ("rows", c_int64), ("dim", c_int32), ("ffn", c_int32), ("vocab", c_int64),
        ("num_q_heads", c_int32), ("num_kv_heads", c_int32), ("head_dim", c_int32), ("max_seq", c_int32),
        ("num_seqs", c_int32), ("eps", c_float), ("theta", c_double),
        ("ids", c_void_p), ("embed", c_void_p), ("hidden", c_void_p), ("attn_out", c_void_p), ("w_attn", c_void_p),
        ("y_attn", c_void_p), ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("positions", c_void_p),
        ("seq_ids", c_void_p), ("k_cache", c_void_p), ("v_cache", c_void_p), ("rope_table", c_void_p),
        ("rope_table_len", c_int32), ("ffn_out", c_void_p), ("w_ffn", c_void_p), ("y_ffn", c_void_p),
        ("gate", c_void_p), ("up", c_void_p), ("act", c_void_p),
    ]


# name -> (restype, argtypes). Every symbol include/bm_layer_ops.h declares.
SIGNATURES = {
    "bm_status_string": (c_char_p, [c_int]),
    "bm_abi_version": (c_int, []),
    "bm_last_error_message": (c_char_p, []),
    "bm_status_read": (c_int, [c_void_p, P_INT32, c_void_p]),
    "bm_embed_gather": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int,
                                c_void_p, c_void_p]),
    "bm_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float, c_int64, c_int64, c_int,
                           c_void_p]),
    "bm_add_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float, c_int,
                               c_void_p]),
    "bm_add": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "bm_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "bm_rope_table_fill": (c_int, [c_void_p, c_int32, c_int32, c_double, c_void_p]),
    "bm_rope_table_create": (c_int, [c_int32, c_int32, c_double, ctypes.POINTER(c_void_p)]),
    "bm_rope_table_destroy": (c_int, [c_void_p]),
    "bm_rope_kv_store": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_int32, c_double, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32,
                                 c_int, c_void_p, c_void_p]),
    "bm_rope": (c_int, [c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_double, c_int64, c_int32,
                        c_int32, c_int32, c_int, c_void_p, c_void_p]),
    "bm_kv_store": (c_int, [c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_int64, c_int32, c_int32, c_int32,
                            c_int32, c_int, c_void_p, c_void_p]),
    "bm_decode_attention_workspace_size": (c_int, [c_int64, c_int32, c_int32, c_int32, c_int32,
                                                   ctypes.POINTER(ctypes.c_size_t)]),
    "bm_gemm_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_int32, c_int, c_void_p,
                               c_void_p]),
    "bm_gemm": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_int32, c_int, c_void_p, c_void_p]),
    "bm_gemm_shared_a": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int64, c_int32, c_int, c_void_p,
                                 c_void_p]),
    "bm_rmsnorm_gemm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_int32, c_int32, c_int64, c_int32, c_int, c_void_p, c_void_p]),
    "bm_rope_kv_decode_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32,
                                            c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int64, c_int32, c_int32,
                                            c_int32, c_int32, c_int32, c_float, c_void_p, ctypes.c_size_t, c_int,
                                            c_void_p, c_void_p]),
    "bm_softmax": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p]),
    "bm_decode_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int64,
                                    c_int32, c_int32, c_int32, c_int32, c_int32, c_float, c_void_p, ctypes.c_size_t,
                                    c_int, c_void_p, c_void_p]),
    "bm_decode_attention_static_scratch": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                                   c_int32, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32,
                                                   c_float, c_int, c_void_p, c_void_p]),
    "bm_kv_cache_create": (c_int, [c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int,
                                   ctypes.POINTER(c_void_p)]),
    "bm_kv_cache_destroy": (c_int, [c_void_p]),
    "bm_kv_cache_layer": (c_int, [c_void_p, c_int32, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p)]),
    "bm_kv_cache_seq_len": (c_int, [c_void_p, c_int32, P_INT32]),
    "bm_kv_cache_reset": (c_int, [c_void_p, c_int32]),
    "bm_kv_cache_append": (c_int, [c_void_p, c_void_p, c_int64, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p),
                                   c_void_p]),
    "bm_selftest_bounded_wait": (c_int, [c_int64, c_void_p, c_void_p, c_void_p]),
    "bm_layer_step": (c_int, [ctypes.POINTER(LayerStepC), c_int, c_void_p, c_void_p]),
}

_lock = threading.Lock()
_lib = None


class BMError(RuntimeError):
    """A non-zero bm_status_t from the C ABI, with the library's message."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} [{status_name(status)}]")
        self.status = status


def status_name(status: int) -> str:
    return {BM_OK: "BM_OK", BM_ERR_INVALID_ARGUMENT: "BM_ERR_INVALID_ARGUMENT", BM_ERR_CUDA: "BM_ERR_CUDA",
            BM_ERR_DEVICE: "BM_ERR_DEVICE"}.get(status, f"BM_ERR_{status}")


def lib_path() -> str:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Loads the library once; raises if it is missing (no fallback path)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build the sm_100a kernels first "
                    "(python -m baremetalinferenceengine_b200.build)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
        return _lib


def check(status: int) -> None:
    if status != BM_OK:
        msg = load().bm_last_error_message()
        raise BMError(status, msg.decode() if msg else "")

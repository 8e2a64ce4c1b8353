"""Host-side API over the C ABI, on torch CUDA tensors (torch provides device
memory and streams; every op runs in ``libbm_layer_ops.so``).

Two layers, mirroring the reference:

* ``launch_*`` — the reference's single-token fp32 launch functions
  (include/kernels.cuh:9,15,29,32,36) with the same names, argument order and
  meaning; tensors stand in for the raw device pointers. Where the reference
  exits the process through CUDA_CHECK, these raise :class:`BMError`.
* batched ops — ``embed_gather``, ``rmsnorm``, ``add_rmsnorm``, ``swiglu``,
  ``add``, ``rope``, ``rope_kv_store``, ``kv_store`` over many rows, fp32 or
  bf16, on the current torch stream of the tensors' device.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from ._lib import BMError, check, load  # noqa: F401  (re-exported)

_DTYPES = {torch.float32: _lib.BM_F32, torch.bfloat16: _lib.BM_BF16}


def bm_dtype(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, f"unsupported dtype {t.dtype} (float32 or bfloat16)") from None


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    if t is None:
        return None
    if not t.is_cuda:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "tensor is not on a CUDA device")
    return t.data_ptr()


def _dev(t: torch.Tensor) -> torch.device:
    """The tensor's CUDA device; a CPU tensor is an argument error (no CPU path)."""
    if not t.is_cuda:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "tensor is not on a CUDA device")
    return t.device


def _stream(device: torch.device, stream: Optional[torch.cuda.Stream]) -> int:
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return s.cuda_stream


def _dense(t: torch.Tensor, name: str) -> None:
    if not t.is_contiguous():
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, f"{name} must be contiguous")


def _same(ref: torch.Tensor, *others: Optional[torch.Tensor]) -> None:
    for o in others:
        if o is not None and (o.device != ref.device or o.dtype != ref.dtype):
            raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "tensors must share device and dtype")


def _i32(t: Optional[torch.Tensor], name: str) -> None:
    if t is not None and (t.dtype != torch.int32 or not t.is_contiguous() or not t.is_cuda):
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, f"{name} must be a contiguous int32 CUDA tensor")


class DeviceStatus:
    """One int32 device word that kernels OR ``BM_DEVERR_*`` bits into."""

    def __init__(self, device: torch.device | str | int = "cuda"):
        self.word = torch.zeros(1, dtype=torch.int32, device=device)

    @property
    def ptr(self) -> int:
        return self.word.data_ptr()

    def read(self, stream: Optional[torch.cuda.Stream] = None) -> int:
        """Synchronises the stream, returns the bits and clears the word."""
        flags = ctypes.c_int32(0)
        with torch.cuda.device(self.word.device):
            st = load().bm_status_read(self.ptr, ctypes.byref(flags), _stream(self.word.device, stream))
        if st not in (_lib.BM_OK, _lib.BM_ERR_DEVICE):
            check(st)
        return int(flags.value)


class RopeTable:
    """Device (cos, sin) table [max_pos][head_dim/2] of fp32 pairs, filled in fp64."""

    def __init__(self, max_pos: int, head_dim: int, theta: float, device: torch.device | str | int = "cuda",
                 stream: Optional[torch.cuda.Stream] = None):
        self.max_pos, self.head_dim, self.theta = int(max_pos), int(head_dim), float(theta)
        self.data = torch.empty(self.max_pos, self.head_dim // 2, 2, dtype=torch.float32, device=device)
        with torch.cuda.device(self.data.device):
            check(load().bm_rope_table_fill(self.data.data_ptr(), self.max_pos, self.head_dim, self.theta,
                                            _stream(self.data.device, stream)))

    @property
    def ptr(self) -> int:
        return self.data.data_ptr()


# --------------------------------------------------------------------------
# Batched ops
# --------------------------------------------------------------------------

def embed_gather(table: torch.Tensor, ids: torch.Tensor, out: Optional[torch.Tensor] = None,
                 status: Optional[DeviceStatus] = None, stream=None) -> torch.Tensor:
    """out[r] = table[ids[r]] (bit-exact). Bad ids leave rows unwritten and set BAD_ID."""
    _dense(table, "table")
    _i32(ids, "ids")
    rows, (vocab, dim) = ids.numel(), table.shape
    if out is None:
        out = torch.empty(rows, dim, dtype=table.dtype, device=table.device)
    _same(table, out)
    if out.dim() != 2 or out.shape[0] != rows or out.shape[1] != dim or out.stride(1) != 1:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "out must be [rows, dim] with unit inner stride")
    with torch.cuda.device(_dev(table)):
        check(load().bm_embed_gather(_ptr(out), _ptr(table), _ptr(ids), rows, dim, vocab, out.stride(0),
                                     bm_dtype(table), status.ptr if status else None,
                                     _stream(table.device, stream)))
    return out


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5, out: Optional[torch.Tensor] = None,
            stream=None) -> torch.Tensor:
    """Row-wise RMSNorm of x [rows, dim]; ``out=x`` normalises in place."""
    dim = x.shape[-1]
    x2 = x.reshape(-1, dim) if x.is_contiguous() else x
    if x2.dim() != 2 or x2.stride(1) != 1:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "x must be [rows, dim] with unit inner stride")
    if out is None:
        out = torch.empty_like(x)
    out2 = out.reshape(-1, dim) if out.is_contiguous() else out
    _same(x, weight, out)
    if weight.numel() != dim:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "weight must have dim elements")
    with torch.cuda.device(_dev(x)):
        check(load().bm_rmsnorm(_ptr(out2), _ptr(x2), _ptr(weight), x2.shape[0], dim, eps, x2.stride(0),
                                out2.stride(0), bm_dtype(x), _stream(x.device, stream)))
    return out


def add_rmsnorm(residual: torch.Tensor, delta: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5,
                out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """residual += delta (in place); returns rmsnorm(residual) * weight."""
    for t, n in ((residual, "residual"), (delta, "delta")):
        _dense(t, n)
    if residual.shape != delta.shape:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "residual and delta shapes differ")
    dim = residual.shape[-1]
    if out is None:
        out = torch.empty_like(residual)
    _dense(out, "out")
    _same(residual, delta, weight, out)
    with torch.cuda.device(_dev(residual)):
        check(load().bm_add_rmsnorm(_ptr(residual), _ptr(delta), _ptr(weight), _ptr(out), residual.numel() // dim,
                                    dim, eps, bm_dtype(residual), _stream(residual.device, stream)))
    return out


def swiglu(gate: torch.Tensor, up: torch.Tensor, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """out = silu(gate) * up, element-wise."""
    _dense(gate, "gate")
    _dense(up, "up")
    if out is None:
        out = torch.empty_like(gate)
    _dense(out, "out")
    _same(gate, up, out)
    if gate.numel() != up.numel() or out.numel() != gate.numel():
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "gate, up and out sizes differ")
    with torch.cuda.device(_dev(gate)):
        check(load().bm_swiglu(_ptr(out), _ptr(gate), _ptr(up), gate.numel(), bm_dtype(gate),
                               _stream(gate.device, stream)))
    return out


def add(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """out = a + b, element-wise (out may be a or b)."""
    _dense(a, "a")
    _dense(b, "b")
    if out is None:
        out = torch.empty_like(a)
    _dense(out, "out")
    _same(a, b, out)
    if a.numel() != b.numel() or out.numel() != a.numel():
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "a, b and out sizes differ")
    with torch.cuda.device(_dev(a)):
        check(load().bm_add(_ptr(out), _ptr(a), _ptr(b), a.numel(), bm_dtype(a), _stream(a.device, stream)))
    return out


def gemm_swiglu(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, out: Optional[torch.Tensor] = None,
                status: Optional[DeviceStatus] = None, stream=None) -> torch.Tensor:
    """out = silu(x @ w_gate) * (x @ w_up): x [rows, dim], w_gate and w_up [dim, hidden]
    (the reference's [in][out] weight layout). bf16 on the tensor cores; fp32 on CUDA
    cores (the SwiGLU of bm_swiglu applied to the reduced products)."""
    for t, name in ((x, "x"), (w_gate, "w_gate"), (w_up, "w_up")):
        _dense(t, name)
    if x.dim() != 2 or w_gate.dim() != 2 or w_gate.shape != w_up.shape or w_gate.shape[0] != x.shape[1]:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "need x [rows, dim] and w_gate, w_up [dim, hidden]")
    rows, dim = x.shape
    hidden = w_gate.shape[1]
    if out is None:
        out = torch.empty((rows, hidden), dtype=x.dtype, device=x.device)
    _dense(out, "out")
    _same(x, w_gate, w_up, out)
    if tuple(out.shape) != (rows, hidden):
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "out must be [rows, hidden]")
    with torch.cuda.device(_dev(x)):
        check(load().bm_gemm_swiglu(_ptr(out), _ptr(x), _ptr(w_gate), _ptr(w_up), rows, dim, hidden, bm_dtype(x),
                                    status.ptr if status else None, _stream(x.device, stream)))
    return out


def gemm(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None,
         status: Optional[DeviceStatus] = None, stream=None) -> torch.Tensor:
    """out = a @ b: a [m, k], b [k, n] (launch_gemm's operand layout). bf16 runs on
    the tensor cores; fp32 on CUDA cores (built for few rows)."""
    _dense(a, "a")
    _dense(b, "b")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "need a [m, k] and b [k, n]")
    m, k = a.shape
    n = b.shape[1]
    if out is None:
        out = torch.empty((m, n), dtype=a.dtype, device=a.device)
    _dense(out, "out")
    _same(a, b, out)
    if tuple(out.shape) != (m, n):
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "out must be [m, n]")
    with torch.cuda.device(_dev(a)):
        check(load().bm_gemm(_ptr(out), _ptr(a), _ptr(b), m, n, k, bm_dtype(a), status.ptr if status else None,
                             _stream(a.device, stream)))
    return out


def gemm_shared_a(a: torch.Tensor, bs, outs=None, status: Optional[DeviceStatus] = None, stream=None):
    """[a @ b for b in bs] for one to three weights b [k, n_o] (an attention block's Q,
    K and V projections): fp32 in one launch, bf16 one tensor-core GEMM per weight."""
    _dense(a, "a")
    bs = list(bs)
    if not 1 <= len(bs) <= 3:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "one to three weights")
    if a.dim() != 2:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "need a [m, k]")
    m, k = a.shape
    for b in bs:
        _dense(b, "b")
        if b.dim() != 2 or b.shape[0] != k:
            raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "need every b [k, n]")
    if outs is None:
        outs = [torch.empty((m, b.shape[1]), dtype=a.dtype, device=a.device) for b in bs]
    outs = list(outs)
    for b, out in zip(bs, outs):
        _dense(out, "out")
        if tuple(out.shape) != (m, b.shape[1]):
            raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "every out must be [m, n]")
    _same(a, *bs, *outs)
    count = len(bs)
    c_arr = (ctypes.c_void_p * count)(*[_ptr(o) for o in outs])
    b_arr = (ctypes.c_void_p * count)(*[_ptr(b) for b in bs])
    n_arr = (ctypes.c_int32 * count)(*[b.shape[1] for b in bs])
    with torch.cuda.device(_dev(a)):
        check(load().bm_gemm_shared_a(c_arr, _ptr(a), b_arr, n_arr, count, m, k, bm_dtype(a),
                                      status.ptr if status else None, _stream(a.device, stream)))
    return outs


def rmsnorm_gemm(h: torch.Tensor, norm_weight: torch.Tensor, bs, d: Optional[torch.Tensor] = None, eps: float = 1e-5,
                 swiglu: bool = False, outs=None, residual_out: Optional[torch.Tensor] = None,
                 normed: Optional[torch.Tensor] = None, status: Optional[DeviceStatus] = None, stream=None):
    """The norm before a projection and the projection: y = rmsnorm(h + d) * norm_weight
    (d optional), then [y @ b for b in bs] (one to three weights), or with swiglu
    (bs = [w_gate, w_up]) the one output silu(y @ w_gate) * (y @ w_up). residual_out,
    when given with d, receives h + d. fp32 rows that fit run as one launch."""
    _dense(h, "h")
    bs = list(bs)
    if h.dim() != 2:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "need h [m, k]")
    m, k = h.shape
    if (len(bs) != 2) if swiglu else not 1 <= len(bs) <= 3:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "two weights with swiglu, else one to three")
    for b in bs:
        _dense(b, "b")
        if b.dim() != 2 or b.shape[0] != k:
            raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "need every b [k, n]")
    widths = [b.shape[1] for b in bs]
    n_out = 1 if swiglu else len(bs)
    if outs is None:
        outs = [torch.empty((m, widths[o]), dtype=h.dtype, device=h.device) for o in range(n_out)]
    outs = list(outs)
    if len(outs) != n_out:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "one output per product (one with swiglu)")
    for o, out in enumerate(outs):
        _dense(out, "out")
        if tuple(out.shape) != (m, widths[o]):
            raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "every out must be [m, n]")
    if normed is None:
        normed = torch.empty_like(h)
    extra = [t for t in (d, residual_out) if t is not None]
    for t in extra + [normed]:
        _dense(t, "h-shaped tensor")
        if tuple(t.shape) != (m, k):
            raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "d, residual_out and normed must be [m, k]")
    _dense(norm_weight, "norm_weight")
    _same(h, norm_weight, *bs, *outs, normed, *extra)
    count = len(bs)
    c_arr = (ctypes.c_void_p * count)(*([_ptr(o) for o in outs] + [None] * (count - len(outs))))
    b_arr = (ctypes.c_void_p * count)(*[_ptr(b) for b in bs])
    n_arr = (ctypes.c_int32 * count)(*widths)
    with torch.cuda.device(_dev(h)):
        check(load().bm_rmsnorm_gemm(c_arr, _ptr(h), _ptr(d), _ptr(norm_weight), eps,
                                     _ptr(residual_out), _ptr(normed), b_arr,
                                     n_arr, count, int(swiglu), m, k, bm_dtype(h), status.ptr if status else None,
                                     _stream(h.device, stream)))
    return outs


def softmax(x: torch.Tensor, size: Optional[int] = None, num_vectors: int = 1, stride: Optional[int] = None,
            stream=None) -> torch.Tensor:
    """In place: num_vectors vectors of `size` elements, `stride` apart, each
    replaced by exp(x - max) / sum exp(x - max) (defaults: x as one vector)."""
    _dense(x, "x")
    size = x.numel() if size is None else size
    stride = size if stride is None else stride
    if num_vectors > 0 and size > 0 and (num_vectors - 1) * stride + size > x.numel():
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "vectors reach past x")
    with torch.cuda.device(_dev(x)):
        check(load().bm_softmax(_ptr(x), size, num_vectors, stride, bm_dtype(x), _stream(x.device, stream)))
    return x


def _positions(positions, rows):
    if isinstance(positions, int):
        return None, positions
    _i32(positions, "positions")
    if positions.numel() != rows:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "positions must have one entry per row")
    return positions, 0


def rope_kv_store(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, positions, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, table: Optional[RopeTable] = None, theta: float = 10000.0,
                  seq_ids: Optional[torch.Tensor] = None, status: Optional[DeviceStatus] = None,
                  stream=None) -> None:
    """Rotates q [rows, Hq, hd] in place; writes rotated k and raw v into the caches
    [num_seqs, Hkv, max_seq, hd] at (seq_ids[r], positions[r]). ``positions`` is an
    int32 tensor or an int pos0 (token r at pos0 + r)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _dense(t, n)
    _same(q, k, v, k_cache, v_cache)
    rows, hq, hd = q.shape[0], q.shape[1], q.shape[2]
    hkv = k.shape[1]
    num_seqs, max_seq = k_cache.shape[0], k_cache.shape[2]
    if k.shape != v.shape or k.shape[0] != rows or k_cache.shape != v_cache.shape or k_cache.shape[1] != hkv:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "q/k/v/cache shapes disagree")
    pos_t, pos0 = _positions(positions, rows)
    _i32(seq_ids, "seq_ids")
    with torch.cuda.device(_dev(q)):
        check(load().bm_rope_kv_store(_ptr(q), _ptr(k), _ptr(v), _ptr(pos_t), pos0, _ptr(seq_ids), _ptr(k_cache),
                                      _ptr(v_cache), table.ptr if table else None,
                                      table.max_pos if table else 0, theta, rows, hq, hkv, hd, max_seq, num_seqs,
                                      bm_dtype(q), status.ptr if status else None, _stream(q.device, stream)))


def rope(q: Optional[torch.Tensor], k: Optional[torch.Tensor], positions, table: Optional[RopeTable] = None,
         theta: float = 10000.0, status: Optional[DeviceStatus] = None, stream=None) -> None:
    """Rotates q [rows, Hq, hd] and k [rows, Hkv, hd] in place (either may be None)."""
    ref = q if q is not None else k
    for t, n in ((q, "q"), (k, "k")):
        if t is not None:
            _dense(t, n)
    _same(ref, q, k)
    rows, hd = ref.shape[0], ref.shape[2]
    pos_t, pos0 = _positions(positions, rows)
    with torch.cuda.device(_dev(ref)):
        check(load().bm_rope(_ptr(q), _ptr(k), _ptr(pos_t), pos0, table.ptr if table else None,
                             table.max_pos if table else 0, theta, rows, q.shape[1] if q is not None else 0,
                             k.shape[1] if k is not None else 0, hd, bm_dtype(ref),
                             status.ptr if status else None, _stream(ref.device, stream)))


def kv_store(cache: torch.Tensor, src: torch.Tensor, positions, seq_ids: Optional[torch.Tensor] = None,
             status: Optional[DeviceStatus] = None, stream=None) -> None:
    """cache [num_seqs, H, max_seq, hd][seq_ids[r], :, positions[r]] = src [rows, H, hd][r]."""
    _dense(cache, "cache")
    _dense(src, "src")
    _same(cache, src)
    rows, h, hd = src.shape
    pos_t, pos0 = _positions(positions, rows)
    _i32(seq_ids, "seq_ids")
    with torch.cuda.device(_dev(src)):
        check(load().bm_kv_store(_ptr(cache), _ptr(src), _ptr(pos_t), pos0, _ptr(seq_ids), rows, h, hd,
                                 cache.shape[2], cache.shape[0], bm_dtype(src), status.ptr if status else None,
                                 _stream(src.device, stream)))


# --------------------------------------------------------------------------
# The reference's launch API (single token, fp32), include/kernels.cuh
# --------------------------------------------------------------------------

def layer_step(ids: torch.Tensor, embed: torch.Tensor, hidden: torch.Tensor, attn_out: torch.Tensor,
               w_attn: torch.Tensor, y_attn: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               positions: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, ffn_out: torch.Tensor,
               w_ffn: torch.Tensor, y_ffn: torch.Tensor, gate: torch.Tensor, up: torch.Tensor, act: torch.Tensor,
               eps: float = 1e-5, table: Optional[RopeTable] = None, theta: float = 10000.0,
               seq_ids: Optional[torch.Tensor] = None, status: Optional[DeviceStatus] = None, stream=None) -> None:
    """One layer step (bm_layer_step): hidden = embed[ids] + attn_out, y_attn =
    rmsnorm(hidden) * w_attn, RoPE on q (in place) and k into k_cache with v into
    v_cache, hidden += ffn_out, y_ffn = rmsnorm(hidden) * w_ffn, act = silu(gate)
    * up. One launch for batches of at most 512 tokens, five otherwise."""
    rows, dim = hidden.shape
    for t, n in ((embed, "embed"), (hidden, "hidden"), (attn_out, "attn_out"), (w_attn, "w_attn"),
                 (y_attn, "y_attn"), (q, "q"), (k, "k"), (v, "v"), (k_cache, "k_cache"), (v_cache, "v_cache"),
                 (ffn_out, "ffn_out"), (w_ffn, "w_ffn"), (y_ffn, "y_ffn"), (gate, "gate"), (up, "up"), (act, "act")):
        _dense(t, n)
    _same(hidden, embed, attn_out, w_attn, y_attn, q, k, v, k_cache, v_cache, ffn_out, w_ffn, y_ffn, gate, up, act)
    _i32(ids, "ids")
    _i32(positions, "positions")
    _i32(seq_ids, "seq_ids")
    ffn = gate.shape[-1]
    shapes_ok = (attn_out.shape == hidden.shape == y_attn.shape == ffn_out.shape == y_ffn.shape
                 and embed.shape[1] == dim and w_attn.numel() == dim and w_ffn.numel() == dim
                 and gate.shape == up.shape == act.shape == (rows, ffn) and ids.numel() == rows
                 and positions.numel() == rows and q.shape[0] == rows and k.shape == v.shape
                 and k.shape[0] == rows and k_cache.shape == v_cache.shape and k_cache.shape[1] == k.shape[1]
                 and (seq_ids is None or seq_ids.numel() == rows))
    if not shapes_ok:
        raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "layer step tensor shapes disagree")
    c = _lib.LayerStepC()
    c.rows, c.dim, c.ffn, c.vocab = rows, dim, ffn, embed.shape[0]
    c.num_q_heads, c.num_kv_heads, c.head_dim = q.shape[1], k.shape[1], q.shape[2]
    c.max_seq, c.num_seqs, c.eps, c.theta = k_cache.shape[2], k_cache.shape[0], eps, theta
    c.ids, c.embed, c.hidden, c.attn_out, c.w_attn, c.y_attn = (_ptr(ids), _ptr(embed), _ptr(hidden), _ptr(attn_out),
                                                                _ptr(w_attn), _ptr(y_attn))
    c.q, c.k, c.v, c.positions, c.seq_ids = _ptr(q), _ptr(k), _ptr(v), _ptr(positions), _ptr(seq_ids)
    c.k_cache, c.v_cache = _ptr(k_cache), _ptr(v_cache)
    c.rope_table = None if table is None else table.ptr
    c.rope_table_len = 0 if table is None else table.max_pos
    c.ffn_out, c.w_ffn, c.y_ffn, c.gate, c.up, c.act = (_ptr(ffn_out), _ptr(w_ffn), _ptr(y_ffn), _ptr(gate),
                                                        _ptr(up), _ptr(act))
    with torch.cuda.device(_dev(hidden)):
        check(load().bm_layer_step(ctypes.byref(c), bm_dtype(hidden), None if status is None else status.ptr,
                                   _stream(hidden.device, stream)))


def _stream_arg(stream) -> int:
    if stream is None or stream == 0:
        return 0
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def launch_rms_norm(out: torch.Tensor, inp: torch.Tensor, weight: torch.Tensor, size: int, eps: float = 1e-5,
                    stream=0) -> None:
    """include/kernels.cuh:9 — one vector of ``size`` floats; out may be inp."""
    with torch.cuda.device(_dev(inp)):
        check(load().bm_rmsnorm(_ptr(out), _ptr(inp), _ptr(weight), 1, size, eps, size, size, _lib.BM_F32,
                                _stream_arg(stream)))


def launch_rope(q: torch.Tensor, k: torch.Tensor, seq_pos: int, head_dim: int, num_heads: int, num_kv_heads: int,
                theta: float = 10000.0, stream=0) -> None:
    """include/kernels.cuh:15 — rotates one token's q and k in place."""
    with torch.cuda.device(_dev(q)):
        check(load().bm_rope(_ptr(q), _ptr(k), None, seq_pos, None, 0, float(theta), 1, num_heads, num_kv_heads,
                             head_dim, _lib.BM_F32, None, _stream_arg(stream)))


def launch_gemm(c: torch.Tensor, a: torch.Tensor, b: torch.Tensor, m: int, n: int, k: int, stream=0) -> None:
    """include/kernels.cuh:20 — c[m][n] = a[m][k] b[k][n], fp32."""
    with torch.cuda.device(_dev(a)):
        check(load().bm_gemm(_ptr(c), _ptr(a), _ptr(b), m, n, k, _lib.BM_F32, None, _stream_arg(stream)))


def launch_softmax_batch(x: torch.Tensor, size: int, num_vectors: int, stride: int, stream=0) -> None:
    """include/kernels.cuh:26 — softmax in place over num_vectors vectors `stride` apart."""
    with torch.cuda.device(_dev(x)):
        check(load().bm_softmax(_ptr(x), size, num_vectors, stride, _lib.BM_F32, _stream_arg(stream)))


def launch_softmax(x: torch.Tensor, size: int, stream=0) -> None:
    """include/kernels.cuh:23 — softmax in place over one vector."""
    launch_softmax_batch(x, size, 1, size, stream)


def launch_swiglu(out: torch.Tensor, gate: torch.Tensor, up: torch.Tensor, size: int, stream=0) -> None:
    """include/kernels.cuh:29 — out = silu(gate) * up."""
    with torch.cuda.device(_dev(gate)):
        check(load().bm_swiglu(_ptr(out), _ptr(gate), _ptr(up), size, _lib.BM_F32, _stream_arg(stream)))


def launch_add(out: torch.Tensor, a: torch.Tensor, b: torch.Tensor, size: int, stream=0) -> None:
    """include/kernels.cuh:32 — out = a + b; out may alias a or b."""
    with torch.cuda.device(_dev(a)):
        check(load().bm_add(_ptr(out), _ptr(a), _ptr(b), size, _lib.BM_F32, _stream_arg(stream)))


def launch_kv_store(cache: torch.Tensor, src: torch.Tensor, seq_pos: int, num_heads: int, head_dim: int,
                    max_seq_len: int, stream=0) -> None:
    """include/kernels.cuh:36 — cache [H][max_seq][hd] at seq_pos = src [H][hd]."""
    with torch.cuda.device(_dev(src)):
        check(load().bm_kv_store(_ptr(cache), _ptr(src), None, seq_pos, None, 1, num_heads, head_dim, max_seq_len,
                                 1, _lib.BM_F32, None, _stream_arg(stream)))


# --------------------------------------------------------------------------
# Batch-aware KV cache (bm_kv_cache_*)
# --------------------------------------------------------------------------

class KVCache:
    """Per-layer K/V caches [num_seqs][kv_heads][max_seq][head_dim] with one length
    per sequence (the reference's KVCache, include/kv_cache.h:10-40, keeps one
    position for the whole cache). Create it with the target device current."""

    def __init__(self, num_layers: int, num_seqs: int, num_kv_heads: int, max_seq: int, head_dim: int,
                 max_tokens: int, dtype: torch.dtype = torch.bfloat16, device=None):
        self.dtype = dtype
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.shape = (num_seqs, num_kv_heads, max_seq, head_dim)
        self.num_layers = num_layers
        handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(load().bm_kv_cache_create(num_layers, num_seqs, num_kv_heads, max_seq, head_dim, max_tokens,
                                            _DTYPES[dtype], ctypes.byref(handle)))
        self._h = handle

    def close(self) -> None:
        if self._h:
            with torch.cuda.device(self.device):
                check(load().bm_kv_cache_destroy(self._h))
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    def layer_ptrs(self, layer: int):
        k, v = ctypes.c_void_p(), ctypes.c_void_p()
        check(load().bm_kv_cache_layer(self._h, layer, ctypes.byref(k), ctypes.byref(v)))
        return k.value, v.value

    def seq_len(self, seq: int) -> int:
        n = ctypes.c_int32()
        check(load().bm_kv_cache_seq_len(self._h, seq, ctypes.byref(n)))
        return n.value

    def reset(self, seq: int = -1) -> None:
        check(load().bm_kv_cache_reset(self._h, seq))

    def append(self, seq_ids, stream=None):
        """Assigns the next position of its sequence to each new token (seq_ids: host
        ints); returns device pointers (positions, seq_ids) for rope_kv_store."""
        import numpy as np

        ids = np.ascontiguousarray(np.asarray(seq_ids, dtype=np.int32))
        pos_p, seq_p = ctypes.c_void_p(), ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(load().bm_kv_cache_append(self._h, ids.ctypes.data if ids.size else None, ids.size,
                                            ctypes.byref(pos_p), ctypes.byref(seq_p),
                                            _stream(self.device, stream)))
        return pos_p.value, seq_p.value, ids.size

    def rope_kv_store(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, appended,
                      table: Optional[RopeTable] = None, theta: float = 10000.0,
                      status: Optional[DeviceStatus] = None, stream=None) -> None:
        """bm_rope_kv_store into `layer` for the tokens of the last append()."""
        pos_p, seq_p, rows = appended
        kc, vc = self.layer_ptrs(layer)
        num_seqs, hkv, max_seq, hd = self.shape
        for t, n in ((q, "q"), (k, "k"), (v, "v")):
            _dense(t, n)
        _same(q, k, v)
        if q.dtype != self.dtype or q.shape[0] != rows or k.shape[1] != hkv or q.shape[2] != hd:
            raise BMError(_lib.BM_ERR_INVALID_ARGUMENT, "q/k/v do not match the cache or the appended tokens")
        with torch.cuda.device(_dev(q)):
            check(load().bm_rope_kv_store(_ptr(q), _ptr(k), _ptr(v), pos_p, 0, seq_p, kc, vc,
                                          table.ptr if table else None, table.max_pos if table else 0, theta,
                                          rows, q.shape[1], hkv, hd, max_seq, num_seqs, bm_dtype(q),
                                          status.ptr if status else None, _stream(q.device, stream)))

    def views(self, layer: int):
        """Layer `layer`'s K and V caches as torch tensors viewing the cache's
        memory (no copy; valid while the cache lives)."""
        typestr = "<f4" if self.dtype == torch.float32 else "<i2"
        out = []
        for p in self.layer_ptrs(layer):
            arr = _DeviceArray(p, self.shape, typestr)
            t = torch.as_tensor(arr, device=self.device)
            out.append(t if self.dtype == torch.float32 else t.view(torch.bfloat16))
        return out


class _DeviceArray:
    """A raw device allocation described by __cuda_array_interface__ (v3)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}

"""TEST INFRASTRUCTURE: the oracle as the checker of one layer step at full size.

A layer step of the benchmarked workloads is 131072 tokens of dim 8192; the
oracle (bm_oracle.c: the reference's double-precision check loops,
tests/kernel_tests.cu:75-79, 122, 175-187, 206, 223-226, and the embedding row
copy of src/execution_engine.cu:98-99) cannot run every row in seconds. So the
check compares a set of SAMPLED rows with the oracle, chosen where a kernel at
that size could go wrong:

* the first and the last row of the step;
* the rows on either side of each kernel's first grid-stride wrap (the
  launch formulas are mirrored in :func:`wrap_rows`; a kernel that skipped its
  later trips would fail there);
* for SwiGLU, the row holding flat element 2^31 (int32 overflow of an index);
* a seeded random spread over all rows.

Usage: ``s = StepSample(b, rows)`` BEFORE the step (it snapshots the inputs the
step overwrites: q is rotated in place), run the step, then ``s.check()``.
Only tests and bench.py's post-timing check import this module.
"""
from __future__ import annotations

import numpy as np

from . import oracle as orc


def _np(t):
    """torch tensor -> numpy for the oracle (bf16 as uint16 bits)."""
    import torch

    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def wrap_rows(shape, sm_count: int) -> dict:
    """First row of each kernel's second grid-stride trip, from the launch formulas
    (None when one trip covers the step):
    gather        csrc/gather.cu: 256-thread blocks, a row group of g threads
                  (g doubles from 32 while g*4 < 16-byte vectors per row), grid
                  capped at sm_count * 8 * 64 blocks;
    add_rmsnorm   csrc/rmsnorm.cu pick_shape/launch_vec: G threads per row
                  (vpt 4 up to 1024 vectors, 8 above), max(G, 256/G*G)-thread
                  blocks, grid capped at sm_count * (2048/block) * 64;
    rope_kv_store csrc/rope_kv.cu launch_typed: one warp per token, 8 per block,
                  grid capped at sm_count * 16 blocks;
    swiglu        csrc/elementwise.cu launch: 256 threads x 4 vectors of 16 bytes
                  a block per trip, grid capped at sm_count * 8 * 16 blocks
                  (returned as the row holding the first element of trip 2)."""
    es, R, D = shape.es, shape.rows, shape.dim
    out = {}
    nv = D * es // 16
    g = 32
    while g < 256 and g * 4 < nv:
        g *= 2
    per_trip = sm_count * 8 * 64 * (256 // g)
    out["embed_gather"] = per_trip if per_trip < R else None
    if nv <= 32:
        group = 32
    elif nv <= 64:
        group = 32
    elif nv <= 1024:
        group = ((nv + 3) // 4 + 31) // 32 * 32
    else:
        group = ((nv + 7) // 8 + 31) // 32 * 32
    block = group if group >= 256 else 256 // group * group
    per_trip = sm_count * (2048 // block) * 64 * (block // group)
    out["add_rmsnorm"] = per_trip if per_trip < R else None
    per_trip = sm_count * 16 * 8
    out["rope_kv_store"] = per_trip if (shape.kind == "layer" and per_trip < R) else None
    elems = sm_count * 8 * 16 * 256 * 4 * (16 // es)
    out["swiglu"] = elems // shape.ffn if elems < R * shape.ffn else None
    return out


def sample_rows(shape, sm_count: int, random_rows: int = 32, seed: int = 0, limit: int | None = None) -> np.ndarray:
    """Sorted unique rows to compare with the oracle (see the module docstring).
    `limit` restricts them to [0, limit) (a rank's own rows)."""
    R = shape.rows if limit is None else min(limit, shape.rows)
    want = {0, R - 1}
    for r in wrap_rows(shape, sm_count).values():
        if r is not None:
            want.update((r - 1, r, r + 1))
    e31 = (1 << 31) // shape.ffn
    if e31 < R:
        want.update((e31, e31 + 1))
    rng = np.random.default_rng(seed)
    want.update(rng.integers(0, R, size=random_rows).tolist())
    return np.array(sorted(r for r in want if 0 <= r < R), np.int64)


class StepSample:
    """Snapshot of the sampled rows' inputs of one LayerBuffers step, taken before
    the step; check() compares the step's outputs at those rows with the oracle."""

    def __init__(self, b, rows: np.ndarray):
        import torch

        self.b = b
        self.rows = np.asarray(rows, np.int64)
        idx = torch.from_numpy(self.rows).to(b.device)
        self.idx = idx
        s = b.shape
        self.layer = s.kind == "layer"
        take = lambda t: _np(t.index_select(0, idx))  # noqa: E731
        self.ids = _np(b.ids.index_select(0, idx)).astype(np.int32)
        uniq, inv = np.unique(self.ids, return_inverse=True)
        self.embed_rows = _np(b.embed.index_select(0, torch.from_numpy(uniq.astype(np.int64)).to(b.device)))
        self.local_ids = inv.astype(np.int32)
        self.gate, self.up = take(b.gate), take(b.up)
        if self.layer:
            self.attn_out, self.ffn_out = take(b.attn_out), take(b.ffn_out)
            self.w_attn, self.w_ffn = _np(b.w_attn), _np(b.w_ffn)
            self.q, self.k, self.v = take(b.q), take(b.k), take(b.v)
            self.positions = _np(b.positions.index_select(0, idx)).astype(np.int32)
            self.seq_ids = _np(b.seq_ids.index_select(0, idx)).astype(np.int32)

    def check(self) -> dict:
        """Per output: worst error in the reference's metric |got - want| / (1 + |want|)
        (tests/kernel_tests.cu:40), or bit equality for the copies. 'ok' is True when
        every float output is within the tolerance (fp32 1e-5, bf16 1e-2) and every
        copy is bit-exact."""
        import torch

        b, s, idx = self.b, self.b.shape, self.idx
        tol = 1e-2 if s.es == 2 else 1e-5
        res = {"rows": int(self.rows.size), "tolerance": tol}
        exact, errs = {}, {}
        h0, bad = orc.gather(self.embed_rows, self.local_ids)
        assert bad == 0
        got_hidden = _np(b.hidden.index_select(0, idx))
        if self.layer:
            h1, y_attn = orc.add_rmsnorm(h0, self.attn_out, self.w_attn, s.eps)
            h2, y_ffn = orc.add_rmsnorm(h1, self.ffn_out, self.w_ffn, s.eps)
            exact["hidden"] = bool(np.array_equal(got_hidden, h2))
            errs["y_attn"] = orc.worst_error(_np(b.y_attn.index_select(0, idx)), y_attn)
            errs["y_ffn"] = orc.worst_error(_np(b.y_ffn.index_select(0, idx)), y_ffn)
            errs["q"] = orc.worst_error(_np(b.q.index_select(0, idx)), orc.rope(self.q, self.positions, s.theta))
            if s.positions == "tiled":  # every (sequence, position) slot written by exactly one row
                seq = torch.from_numpy(self.seq_ids.astype(np.int64)).to(b.device)
                pos = torch.from_numpy(self.positions.astype(np.int64)).to(b.device)
                k_slots = _np(b.k_cache[seq, :, pos, :])
                v_slots = _np(b.v_cache[seq, :, pos, :])
                errs["k_cache"] = orc.worst_error(k_slots, orc.rope(self.k, self.positions, s.theta))
                exact["v_cache"] = bool(np.array_equal(v_slots, self.v))
        else:
            exact["hidden"] = bool(np.array_equal(got_hidden, h0))
        errs["act"] = orc.worst_error(_np(b.act.index_select(0, idx)), orc.swiglu(self.gate, self.up))
        res["worst_error"] = {k: float(v) for k, v in errs.items()}
        res["bit_exact"] = exact
        res["ok"] = all(v <= tol for v in errs.values()) and all(exact.values())
        return res

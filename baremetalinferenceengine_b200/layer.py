"""One layer's memory-bound ops over a batch of tokens ("a layer step").

The in-scope half of ExecutionEngine::run_layers (src/execution_engine.cu:89-128),
batched over rows and with the adds fused into the norms that follow them:

    hidden        = embed[ids]                                  (:98-99)
    hidden       += attn_out;  y_attn = rmsnorm(hidden) * w_attn (:118 + :109/:121)
    q             = rope(q); k_cache/v_cache[seq, :, pos] = rope(k), v   (:113-115)
    hidden       += ffn_out;   y_ffn  = rmsnorm(hidden) * w_ffn  (:126 + :121/:80)
    act           = silu(gate) * up                             (:124)

The GEMMs between these ops are outside the path: their outputs (attn_out, q,
k, v, ffn_out, gate, up) are inputs here. :data:`WORKLOADS` holds the token
layouts and model shapes the kernels are measured on; :class:`LayerBuffers`
allocates and seeds one step's device buffers; :func:`run_step` issues the
launches through the C ABI (:func:`step_launchers` gives them one by one).
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import torch

from . import ops


@dataclasses.dataclass(frozen=True)
class LayerShape:
    name: str
    rows: int          # tokens per step (per GPU)
    dim: int
    hq: int
    hkv: int
    hd: int
    ffn: int
    vocab: int
    theta: float
    max_seq: int
    num_seqs: int
    dtype: torch.dtype
    eps: float = 1e-5
    positions: str = "tiled"  # "tiled": pos = r mod max_seq, seq = r // max_seq; "uniform": pos ~ U[0, max_seq)
    description: str = ""
    kind: str = "layer"  # "layer": the five ops; "stress": Zipf-id gather + SwiGLU with +-20 outliers

    @property
    def es(self) -> int:
        return 4 if self.dtype == torch.float32 else 2

    @property
    def fused(self) -> bool:
        """Whether the step runs as one launch (bm_layer_step's single-launch form:
        a layer step of at most FUSED_MAX_ROWS tokens)."""
        return self.kind == "layer" and self.rows <= FUSED_MAX_ROWS

    def bytes_per_row(self) -> dict:
        """Algorithmic HBM bytes per token for each kernel: every input element read
        once and every output element written once (weights, the RoPE table and
        the embedding rows' reuse are not counted). layer_step is the single-launch
        step: the embedding row, both deltas read, y_attn, y_ffn and hidden written
        once (the residual never round-trips), RoPE + K/V and SwiGLU as above."""
        es = self.es
        b = {
            "embed_gather": 2 * self.dim * es + 4,
            "add_rmsnorm": 4 * self.dim * es,  # read residual + delta, write residual + out
            "rope_kv_store": (2 * self.hq * self.hd + 2 * self.hkv * self.hd + 2 * self.hkv * self.hd) * es + 8,
            "swiglu": 3 * self.ffn * es,
        }
        b["layer_step"] = 6 * self.dim * es + 4 + b["rope_kv_store"] + b["swiglu"]
        return b

    def op_bytes(self) -> int:
        """Algorithmic bytes of the step's five ops as separate kernels (the
        workload's metric, whichever way the step is launched)."""
        b = self.bytes_per_row()
        if self.kind == "stress":
            return (b["embed_gather"] + b["swiglu"]) * self.rows
        return (b["embed_gather"] + 2 * b["add_rmsnorm"] + b["rope_kv_store"] + b["swiglu"]) * self.rows

    def step_kernels(self) -> list:
        """(kernel, algorithmic bytes per launch) in launch order for one step."""
        b = self.bytes_per_row()
        r = self.rows
        if self.fused:
            return [("layer_step", b["layer_step"] * r)]
        if self.kind == "stress":
            return [("embed_gather", b["embed_gather"] * r), ("swiglu", b["swiglu"] * r)]
        return [("embed_gather", b["embed_gather"] * r), ("add_rmsnorm_attn", b["add_rmsnorm"] * r),
                ("rope_kv_store", b["rope_kv_store"] * r), ("add_rmsnorm_ffn", b["add_rmsnorm"] * r),
                ("swiglu", b["swiglu"] * r)]

    def step_bytes(self) -> int:
        return self.op_bytes()

    def with_rows(self, rows: int) -> "LayerShape":
        return dataclasses.replace(self, rows=rows)


# Layer steps of at most this many tokens run as one launch (bm_layer_step; the
# library's BM_STEP_FUSED_MAX_ROWS).
FUSED_MAX_ROWS = 512

# Synthetic workloads (seeded; no dataset): the model shapes and token layouts the
# kernels are measured on.
WORKLOADS = {
    "tinyllama_fp32": LayerShape(
        "tinyllama_fp32", rows=256, dim=288, hq=6, hkv=6, hd=48, ffn=768, vocab=32000, theta=1e4, max_seq=256,
        num_seqs=1, dtype=torch.float32,
        description="tinyllama-15M-shaped layer, fp32, 256 tokens at positions 0..255"),
    "llama8b_decode_bf16": LayerShape(
        "llama8b_decode_bf16", rows=64, dim=4096, hq=32, hkv=8, hd=128, ffn=14336, vocab=128256, theta=5e5,
        max_seq=8192, num_seqs=64, dtype=torch.bfloat16, positions="uniform",
        description="Llama-3-8B decode: 64 tokens of 64 sequences, positions U[0,8192)"),
    "llama8b_decode_fp32": LayerShape(
        "llama8b_decode_fp32", rows=64, dim=4096, hq=32, hkv=8, hd=128, ffn=14336, vocab=128256, theta=5e5,
        max_seq=8192, num_seqs=64, dtype=torch.float32, positions="uniform",
        description="Llama-3-8B decode, fp32"),
    "llama8b_prefill_bf16": LayerShape(
        "llama8b_prefill_bf16", rows=32768, dim=4096, hq=32, hkv=8, hd=128, ffn=14336, vocab=128256, theta=5e5,
        max_seq=8192, num_seqs=4, dtype=torch.bfloat16,
        description="Llama-3-8B prefill: 4 sequences x 8192 tokens"),
    "swiglu_stress_bf16": LayerShape(
        "swiglu_stress_bf16", rows=65536, dim=4096, hq=32, hkv=8, hd=128, ffn=14336, vocab=128256, theta=5e5,
        max_seq=8192, num_seqs=8, dtype=torch.bfloat16, kind="stress",
        description="SwiGLU stress: 65536 tokens x FFN 14336 with 1% of gate/up at +-20, and a gather of "
                    "65536 Zipf(1.1) ids over vocab 128256 (dim 4096)"),
    "llama70b_bf16": LayerShape(
        "llama70b_bf16", rows=131072, dim=8192, hq=64, hkv=8, hd=128, ffn=28672, vocab=128256, theta=5e5,
        max_seq=8192, num_seqs=16, dtype=torch.bfloat16,
        description="Llama-3-70B: 131072 tokens = 16 sequences x 8192 positions"),
}


def _generator(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


class LayerBuffers:
    """Device buffers of one layer step, seeded N(0,1) activations, 1+N(0,0.02)
    norm weights, N(0,0.02) embedding table, uniform token ids."""

    def __init__(self, shape: LayerShape, device, seed: int = 0, row_offset: int = 0, with_table: bool = True,
                 packed: bool = False):
        s = shape
        self.shape = s
        self.device = torch.device(device)
        dt = s.dtype
        g = _generator(self.device, seed)

        def randn(*size, scale=1.0, offset=0.0):
            t = torch.randn(*size, generator=g, device=self.device, dtype=torch.float32)
            if scale != 1.0:
                t.mul_(scale)
            if offset != 0.0:
                t.add_(offset)
            return t.to(dt)

        R, D = s.rows, s.dim
        self.embed = randn(s.vocab, D, scale=0.02)
        if s.kind == "stress":
            # Zipf(1.1) over the vocabulary by inverse CDF: heavy repeats of the first ids
            rank = torch.arange(1, s.vocab + 1, device=self.device, dtype=torch.float64)
            cdf = torch.cumsum(rank.pow(-1.1), 0)
            u = torch.rand(R, generator=g, device=self.device, dtype=torch.float64) * cdf[-1]
            self.ids = torch.searchsorted(cdf, u).clamp_(max=s.vocab - 1).to(torch.int32)
        else:
            self.ids = torch.randint(0, s.vocab, (R,), generator=g, device=self.device, dtype=torch.int32)
        if s.positions == "uniform":
            self.positions = torch.randint(0, s.max_seq, (R,), generator=g, device=self.device, dtype=torch.int32)
            self.seq_ids = (torch.arange(R, device=self.device, dtype=torch.int32) % s.num_seqs).contiguous()
        else:
            glob = torch.arange(row_offset, row_offset + R, device=self.device, dtype=torch.int64)
            self.positions = (glob % s.max_seq).to(torch.int32)
            seq = glob // s.max_seq - row_offset // s.max_seq
            self.seq_ids = (seq % s.num_seqs).to(torch.int32)
        self.hidden = torch.empty(R, D, dtype=dt, device=self.device)
        self.attn_out = randn(R, D)
        self.w_attn = randn(D, scale=0.02, offset=1.0)
        self.y_attn = torch.empty(R, D, dtype=dt, device=self.device)
        self.q = randn(R, s.hq, s.hd)
        self.k = randn(R, s.hkv, s.hd)
        self.v = randn(R, s.hkv, s.hd)
        self.k_cache = torch.zeros(s.num_seqs, s.hkv, s.max_seq, s.hd, dtype=dt, device=self.device)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.ffn_out = randn(R, D)
        self.w_ffn = randn(D, scale=0.02, offset=1.0)
        self.y_ffn = torch.empty(R, D, dtype=dt, device=self.device)
        self.gate = randn(R, s.ffn)
        self.up = randn(R, s.ffn)
        if s.kind == "stress":  # 1% of entries at +-20: silu saturates on both sides
            for t in (self.gate, self.up):
                mask = torch.rand(t.shape, generator=g, device=self.device) < 0.01
                sign = torch.where(torch.rand(t.shape, generator=g, device=self.device) < 0.5, -20.0, 20.0)
                t[mask] = sign[mask].to(dt)
        self.act = torch.empty(R, s.ffn, dtype=dt, device=self.device)
        self.table = ops.RopeTable(s.max_seq, s.hd, s.theta, self.device) if with_table else None
        self.status = ops.DeviceStatus(self.device)
        self.arena = None
        if packed:
            self._pack()

    # Arena order: tensors only read, then those read and written, then those only
    # written, each at a 256-byte boundary; so a step's inputs are one contiguous
    # range ([0, in_end)) and its outputs another ([out_start, end)).
    def _arena_groups(self):
        ins, out = self.inputs(), self.outputs()
        both = tuple(n for n in ins if n in out)
        return tuple(n for n in ins if n not in both), both, tuple(n for n in out if n not in both)

    def _pack(self) -> None:
        """Moves the step's inputs and outputs into one device allocation (views at
        256-byte boundaries), so a host-buffer step copies in one range and back
        one range."""
        only_in, both, only_out = self._arena_groups()
        offsets, off = {}, 0
        for n in only_in + both + only_out:
            t = getattr(self, n)
            offsets[n] = off
            off += -(-t.numel() * t.element_size() // 256) * 256
        arena = torch.empty(off, dtype=torch.uint8, device=self.device)
        self.arena_offsets = offsets
        for n, o in offsets.items():
            t = getattr(self, n)
            view = arena[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
            view.copy_(t)
            setattr(self, n, view)
        self.arena = arena
        last_in = (only_in + both)[-1]
        self.in_end = offsets[last_in] + getattr(self, last_in).numel() * getattr(self, last_in).element_size()
        self.out_start = offsets[(both + only_out)[0]]

    def with_arena(self, arena: torch.Tensor) -> "LayerBuffers":
        """A shallow copy whose step inputs and outputs are views into `arena` (same
        size and layout as self.arena); everything else (the table, weights, caches,
        status word) is shared. Two arenas let one step's outputs go back while the
        next step's inputs come in."""
        import copy

        if self.arena is None or arena.numel() != self.arena.numel():
            raise ValueError("with_arena needs a packed LayerBuffers and an arena of the same size")
        other = copy.copy(self)
        for n, o in self.arena_offsets.items():
            t = getattr(self, n)
            setattr(other, n, arena[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape))
        other.arena = arena
        return other

    def inputs(self) -> tuple:
        """Tensors an end-to-end (host-buffer) step copies in, every step."""
        if self.shape.kind == "stress":
            return ("ids", "gate", "up")
        return ("ids", "positions", "seq_ids", "attn_out", "q", "k", "v", "ffn_out", "gate", "up")

    def outputs(self) -> tuple:
        """Tensors an end-to-end step copies back, every step (the KV cache stays on the device)."""
        if self.shape.kind == "stress":
            return ("hidden", "act")
        return ("hidden", "y_attn", "q", "y_ffn", "act")

    def nbytes(self, names) -> int:
        return sum(getattr(self, n).numel() * getattr(self, n).element_size() for n in names)


def step_launchers(b: LayerBuffers, stream: Optional[torch.cuda.Stream] = None,
                   rows: Optional[slice] = None) -> list:
    """The step's kernels as (name, launch) pairs in order; each launch issues one
    kernel on `stream` (default: the current stream). `rows` restricts the step
    to a contiguous row range (a chunk). Names match LayerShape.step_kernels."""
    s = b.shape
    sl = rows if rows is not None else slice(0, s.rows)
    st = b.status
    if s.fused:
        return [("layer_step", lambda: ops.layer_step(
            b.ids[sl], b.embed, b.hidden[sl], b.attn_out[sl], b.w_attn, b.y_attn[sl], b.q[sl], b.k[sl], b.v[sl],
            b.positions[sl], b.k_cache, b.v_cache, b.ffn_out[sl], b.w_ffn, b.y_ffn[sl], b.gate[sl], b.up[sl],
            b.act[sl], s.eps, table=b.table, theta=s.theta, seq_ids=b.seq_ids[sl], status=st, stream=stream))]
    gather = ("embed_gather", lambda: ops.embed_gather(b.embed, b.ids[sl], out=b.hidden[sl], status=st,
                                                        stream=stream))
    swiglu = ("swiglu", lambda: ops.swiglu(b.gate[sl], b.up[sl], out=b.act[sl], stream=stream))
    if s.kind == "stress":
        return [gather, swiglu]
    return [
        gather,
        ("add_rmsnorm_attn", lambda: ops.add_rmsnorm(b.hidden[sl], b.attn_out[sl], b.w_attn, s.eps,
                                                     out=b.y_attn[sl], stream=stream)),
        ("rope_kv_store", lambda: ops.rope_kv_store(b.q[sl], b.k[sl], b.v[sl], b.positions[sl], b.k_cache,
                                                    b.v_cache, table=b.table, theta=s.theta,
                                                    seq_ids=b.seq_ids[sl], status=st, stream=stream)),
        ("add_rmsnorm_ffn", lambda: ops.add_rmsnorm(b.hidden[sl], b.ffn_out[sl], b.w_ffn, s.eps,
                                                    out=b.y_ffn[sl], stream=stream)),
        swiglu,
    ]


def run_step(b: LayerBuffers, stream: Optional[torch.cuda.Stream] = None, events: Optional[list] = None,
             rows: Optional[slice] = None) -> int:
    """Issues the step's kernels on `stream` (default: the current stream). With
    `events` (one more than the launches), records one before the first launch
    and one after each. `rows` restricts the step to a row range. Returns the
    number of kernel launches."""
    launchers = step_launchers(b, stream, rows)
    if events is not None:
        events[0].record(stream)
    for i, (_, launch) in enumerate(launchers):
        launch()
        if events is not None:
            events[i + 1].record(stream)
    return len(launchers)

"""Shared test helpers: seeded inputs and torch <-> oracle (numpy) conversion.

Tolerances follow the reference's metric |got - want| / (1 + |want|)
(tests/kernel_tests.cu:36-47): fp32 within 1e-5, bf16 within 1e-2; the gather
and the KV-cache copies are bit-exact.
"""
from __future__ import annotations

import os

import numpy as np
import torch

TOL = {torch.float32: 1e-5, torch.bfloat16: 1e-2}


def to_np(t: torch.Tensor) -> np.ndarray:
    """A CPU numpy view for the oracle: float32, or bf16 as uint16 bits."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float32:
        return t.numpy().copy()
    return t.numpy().copy()


def from_np(a: np.ndarray, device=None) -> torch.Tensor:
    if a.dtype == np.uint16:
        t = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    else:
        t = torch.from_numpy(a.copy())
    return t.to(device) if device is not None else t


def randn(shape, dtype, gen: torch.Generator, scale: float = 1.0, offset: float = 0.0) -> torch.Tensor:
    x = torch.randn(shape, generator=gen, dtype=torch.float32) * scale + offset
    return x.to(dtype)


def gen(seed: int) -> torch.Generator:
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    a, b = a.detach().cpu().contiguous(), b.detach().cpu().contiguous()
    if a.dtype != b.dtype or a.shape != b.shape:
        return False
    if a.dtype in (torch.float32, torch.int32):
        return torch.equal(a.view(torch.int32), b.view(torch.int32))
    return torch.equal(a.view(torch.int16), b.view(torch.int16))


def reference_dir():
    """The reference's source checkout, if present: $BM_REFERENCE_DIR, else a
    `reference` directory beside this repository's. None when neither holds the
    sources (a GPU host has only the prebuilt checkers under oracle/_ref)."""
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for cand in (os.environ.get("BM_REFERENCE_DIR"), os.path.join(os.path.dirname(repo), "reference")):
        if cand and os.path.isdir(os.path.join(cand, "src")):
            return os.path.abspath(cand)
    return None

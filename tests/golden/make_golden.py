"""Writes the golden fixtures in this directory from the reference's own code.

    python tests/golden/make_golden.py

* rope_reference.npz — outputs of the reference's ``reference_rope``
  (tests/kernel_tests.cu:175-187), run from oracle/_ref/libref_cpu.so (the
  reference's unmodified kernel_tests.cu compiled by oracle/Makefile), on seeded
  U[-1,1] inputs at the reference's three test points (position 0, 1 and 37,
  tests/kernel_tests.cu:280-282) and at Llama-3 8B/70B points (theta 5e5,
  head_dim 128, positions up to 8191).
* swiglu_known_answers.npz — the known-answer inputs and outputs of
  tests/kernel_tests.cu:164-173.
* gemm_reference.npz — outputs of the reference's ``reference_gemm``
  (tests/kernel_tests.cu:49-59) at two of its test shapes (16x16x16 and
  128x128x128, :263-264) and at a decode-like and a ragged shape, on U[-1,1]
  inputs rounded to bf16 (so the fp32 inputs the reference sees are exactly the
  bf16 operands of the tensor-core GEMM). Also the gate and up products of a
  small SwiGLU FFN (x, w_gate, w_up) from ``reference_gemm``, for the fused
  GEMM + SwiGLU.

The fixtures are committed so that the GPU host, which has no copy of the
reference, can pin the kernels and the oracle to the reference's outputs.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as orc  # noqa: E402

# (seq_pos, head_dim, heads, theta)
ROPE_POINTS = [
    (0, 48, 6, 10000.0),
    (1, 48, 3, 10000.0),
    (37, 128, 8, 10000.0),
    (255, 48, 6, 10000.0),
    (4095, 128, 32, 500000.0),
    (8191, 128, 8, 500000.0),
    (8191, 128, 64, 500000.0),
]

# (m, n, k): two of the reference's own test_gemm shapes (tests/kernel_tests.cu:263-264),
# one row as in decode, and a shape ragged against the 128 x 256 x 64 tiles
GEMM_SHAPES = [(16, 16, 16), (128, 128, 128), (1, 64, 256), (40, 136, 264)]
SWIGLU_SHAPE = (48, 264, 72)  # rows, dim, hidden


def main() -> int:
    if not orc.ref_available():
        print("oracle/_ref/libref_cpu.so is missing: run `make -C oracle ref` where the reference is present")
        return 1
    rng = np.random.default_rng(20240601)
    arrays = {}
    for n, (pos, hd, heads, theta) in enumerate(ROPE_POINTS):
        x = rng.uniform(-1.0, 1.0, size=(heads, hd)).astype(np.float32)
        arrays[f"x{n}"] = x
        arrays[f"out{n}"] = orc.ref_reference_rope(x, pos, theta)
        arrays[f"meta{n}"] = np.array([pos, hd, heads, theta], dtype=np.float64)
    arrays["count"] = np.array(len(ROPE_POINTS))
    np.savez_compressed(os.path.join(HERE, "rope_reference.npz"), **arrays)

    gate = np.array([-1000.0, -100.0, 0.0, 100.0, 1000.0], np.float32)  # tests/kernel_tests.cu:165
    up = np.full(5, 2.0, np.float32)  # :166
    want = np.array([0.0, 0.0, 0.0, 200.0, 2000.0], np.float32)  # :167
    np.savez_compressed(os.path.join(HERE, "swiglu_known_answers.npz"), gate=gate, up=up, want=want)
    g = {}
    for n, (m, nn, k) in enumerate(GEMM_SHAPES):
        a = orc.f32_to_bf16(rng.uniform(-1.0, 1.0, size=(m, k)).astype(np.float32))
        b = orc.f32_to_bf16(rng.uniform(-1.0, 1.0, size=(k, nn)).astype(np.float32))
        g[f"a{n}"], g[f"b{n}"] = a, b
        g[f"c{n}"] = orc.ref_reference_gemm(orc.bf16_to_f32(a), orc.bf16_to_f32(b))
    g["count"] = np.array(len(GEMM_SHAPES))
    rows, dim, hidden = SWIGLU_SHAPE
    x = orc.f32_to_bf16(rng.uniform(-1.0, 1.0, size=(rows, dim)).astype(np.float32))
    wg = orc.f32_to_bf16(rng.uniform(-0.1, 0.1, size=(dim, hidden)).astype(np.float32))
    wu = orc.f32_to_bf16(rng.uniform(-0.1, 0.1, size=(dim, hidden)).astype(np.float32))
    g["ffn_x"], g["ffn_w_gate"], g["ffn_w_up"] = x, wg, wu
    g["ffn_gate"] = orc.ref_reference_gemm(orc.bf16_to_f32(x), orc.bf16_to_f32(wg))
    g["ffn_up"] = orc.ref_reference_gemm(orc.bf16_to_f32(x), orc.bf16_to_f32(wu))
    np.savez_compressed(os.path.join(HERE, "gemm_reference.npz"), **g)
    print("wrote rope_reference.npz, swiglu_known_answers.npz and gemm_reference.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())

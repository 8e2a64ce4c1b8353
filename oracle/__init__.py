"""TEST INFRASTRUCTURE: the CPU oracle for the layer-op kernels.

Importable only by the tests, the smoke check and the benchmark's CPU-baseline
leg, as the checker (or the timed CPU baseline) — never by the product path.
See :mod:`oracle.oracle` and ``bm_oracle.c``.
"""

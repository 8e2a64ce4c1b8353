"""B200-native (sm_100a) fused transformer-layer kernels of BareMetalInferenceEngine.

The ops (embedding gather, RMSNorm and fused residual-add + RMSNorm, RoPE with
the K/V write into a static KV cache, SwiGLU) live in ``libbm_layer_ops.so``,
built from ``csrc/`` by :mod:`baremetalinferenceengine_b200.build`, behind the C
ABI of ``include/bm_layer_ops.h`` and the reference's own launch signatures
(``include/kernels.cuh``). :mod:`.ops` is the Python host side over torch tensors.
"""
from ._lib import BMError, lib_path, load  # noqa: F401

__all__ = ["BMError", "lib_path", "load"]

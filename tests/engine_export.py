"""Writes a seeded synthetic model in the reference's export format.

The format is the one ModelLoader::load reads (src/weights.cpp:23-93):
model_index.txt ("baremetal-llama 1", key/value settings, "tensors N", then one
"name offset bytes rows cols" line per tensor) and model.bin (fp32 tensors back
to back; 1-D weights as one row; projections stored [in][out]). Tensor names are
the ones ExecutionEngine looks up (src/execution_engine.cu:9-26). No real
checkpoint is available, so the weights are random with shapes of the
tinyllama-15M-sized model: projections N(0, 1/in), norms 1 + N(0, 0.02),
embeddings N(0, 1).
"""
from __future__ import annotations

import os

import numpy as np


def write_export(path: str, dim: int = 288, hidden: int = 768, vocab: int = 32000, layers: int = 6,
                 heads: int = 6, max_seq: int = 256, eps: float = 1e-5, theta: float = 10000.0,
                 seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    specs = [("model.embed_tokens.weight", (vocab, dim), "embed")]
    for layer in range(layers):
        p = f"model.layers.{layer}."
        specs += [(p + "input_layernorm.weight", (1, dim), "norm"),
                  (p + "self_attn.q_proj.weight", (dim, dim), "proj"),
                  (p + "self_attn.k_proj.weight", (dim, dim), "proj"),
                  (p + "self_attn.v_proj.weight", (dim, dim), "proj"),
                  (p + "self_attn.o_proj.weight", (dim, dim), "proj"),
                  (p + "post_attention_layernorm.weight", (1, dim), "norm"),
                  (p + "mlp.gate_proj.weight", (dim, hidden), "proj"),
                  (p + "mlp.up_proj.weight", (dim, hidden), "proj"),
                  (p + "mlp.down_proj.weight", (hidden, dim), "proj")]
    specs += [("model.norm.weight", (1, dim), "norm"), ("lm_head.weight", (dim, vocab), "proj")]
    lines = ["baremetal-llama 1", f"dim {dim}", f"hidden_dim {hidden}", f"vocab_size {vocab}",
             f"num_layers {layers}", f"num_heads {heads}", f"max_seq_len {max_seq}", f"norm_eps {eps}",
             f"rope_theta {theta}", f"tensors {len(specs)}"]
    os.makedirs(path, exist_ok=True)
    offset = 0
    with open(os.path.join(path, "model.bin"), "wb") as f:
        for name, (rows, cols), kind in specs:
            if kind == "norm":
                data = 1.0 + 0.02 * rng.standard_normal((rows, cols))
            elif kind == "embed":
                data = rng.standard_normal((rows, cols))
            else:
                data = rng.standard_normal((rows, cols)) / np.sqrt(rows)
            data = data.astype("<f4")
            f.write(data.tobytes())
            lines.append(f"{name} {offset} {data.size * 4} {rows} {cols}")
            offset += data.size * 4
    with open(os.path.join(path, "model_index.txt"), "w") as f:
        f.write("\n".join(lines) + "\n")
    return {"dim": dim, "vocab": vocab, "layers": layers, "heads": heads, "max_seq": max_seq}

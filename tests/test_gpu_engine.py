"""The drop-in ExecutionEngine on the fused ops (baremetalinferenceengine_b200/engine),
checked with the reference's own programs.

* The reference's tests/logits_test.cu, unmodified, built on this engine
  (engine/_build/logits_test_fused) passes against golden logits that the
  reference's engine and kernels produce for the same seeded synthetic export:
  every position within 0.01, the same next token everywhere, and a reset
  followed by the whole sequence in one forward() call (one batched pass here).
* The reference's src/benchmark.cpp (greedy decode of 100 tokens), unmodified,
  generates the same tokens on three builds: the reference's engine and kernels,
  the reference's engine on this library's layer ops, and this engine.
"""
import json
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle as orc
from tests.engine_export import write_export

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENGINE_BUILD = os.path.join(REPO, "baremetalinferenceengine_b200", "engine", "_build")


def need(path):
    if not os.path.exists(path):
        pytest.fail(f"{path} is missing: build it where the reference's sources are present "
                    "(make -C oracle ref; make -C baremetalinferenceengine_b200/engine)")
    return path


def test_fused_engine_passes_the_reference_logits_test(cuda, tmp_path):
    cfg = write_export(str(tmp_path), seed=21)
    tokens = [int(t) for t in np.random.default_rng(22).integers(0, cfg["vocab"], 48)]
    gold = subprocess.run([need(os.path.join(orc.REF_DIR, "engine_golden_ref")), str(tmp_path)] +
                          [str(t) for t in tokens], capture_output=True, text=True, timeout=600)
    assert gold.returncode == 0, gold.stdout[-2000:] + gold.stderr[-2000:]
    run = subprocess.run([need(os.path.join(ENGINE_BUILD, "logits_test_fused")), str(tmp_path)],
                         capture_output=True, text=True, timeout=600)
    print(run.stdout[-1500:])
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-2000:]
    assert "0 check(s) failed" in run.stdout


def test_reference_benchmark_generates_the_same_tokens_on_every_build(cuda, tmp_path):
    write_export(str(tmp_path), seed=31)
    results = {}
    for name, exe in [("reference", os.path.join(orc.REF_DIR, "benchmark_ref")),
                      ("reference engine + B200 kernels", os.path.join(orc.REF_DIR, "benchmark_dropin")),
                      ("fused engine", os.path.join(ENGINE_BUILD, "benchmark_fused"))]:
        out = tmp_path / (name.split()[0] + str(len(results)) + ".json")
        proc = subprocess.run([need(exe), str(tmp_path), str(out)], capture_output=True, text=True, timeout=900)
        assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-2000:]
        results[name] = json.loads(out.read_text())
    for name, r in results.items():
        print(f"{name:36s} {r['tokens_per_s']:10.1f} tokens/s  ({r['generated_tokens']} greedy tokens)")
    ref_tokens = results["reference"]["tokens"]
    for name, r in results.items():
        assert r["tokens"] == ref_tokens, name

"""Compiles the sm_100a layer-op kernels into the in-tree shared library.

    python -m baremetalinferenceengine_b200.build [--force]

produces ``baremetalinferenceengine_b200/libbm_layer_ops.so`` from ``csrc/*.cu``
with nvcc (``-gencode arch=compute_100a,code=sm_100a``), static cudart, C++17.
Objects go to ``_build/`` at the repository root. A source newer than the
library (or a changed header) triggers a rebuild.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_ROOT = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_ROOT, "include")
BUILD_DIR = os.path.join(REPO_ROOT, "_build", "bm_layer_ops")
LIB_NAME = "libbm_layer_ops.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O3",
    "--expt-relaxed-constexpr",
    "-I" + INCLUDE,
    "-I" + CSRC,
]


def nvcc_path() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build the layer-op kernels")


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith((".h", ".cuh"))]
    return hs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError("command failed:\n  " + " ".join(cmd) + "\n" + proc.stdout)


def build(force: bool = False, verbose: bool = False) -> str:
    """Builds (if needed) and returns the path of libbm_layer_ops.so."""
    nvcc = nvcc_path()
    os.makedirs(BUILD_DIR, exist_ok=True)
    headers = _headers()
    objs = []
    jobs = []
    for src in sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            jobs.append([nvcc] + NVCC_FLAGS + ["-c", src, "-o", obj])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
            for f in [ex.submit(_run, j) for j in jobs]:
                f.result()
            if verbose:
                for j in jobs:
                    print(" ".join(j))
    if force or jobs or _stale(LIB_PATH, objs):
        tmp = LIB_PATH + ".tmp"
        _run([nvcc] + ARCH_FLAGS + ["-shared", "-o", tmp] + objs + ["-lcudart_static", "-lrt", "-ldl", "-lpthread"])
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())

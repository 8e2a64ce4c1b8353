"""pytest configuration: the `gpu` marker and shared fixtures.

Tests marked ``gpu`` need a CUDA device and the built ``libbm_layer_ops.so``;
they fail (not skip) without them, so a GPU run can never pass on a fallback.
Everything else runs on a CPU-only machine.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built sm_100a library")


@pytest.fixture(scope="session")
def cuda():
    import torch

    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    from baremetalinferenceengine_b200 import load

    load()  # raises if the library is missing: no fallback
    return torch.device("cuda", 0)

"""pytest configuration: the `gpu` marker and shared helpers.

Tests marked `gpu` need a CUDA device and the in-tree libalpaca_cuda.so; everything else runs on CPU.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device and the built libalpaca_cuda.so")


@pytest.fixture(scope="session")
def cuda_lib():
    """The loaded product library on a CUDA device; building it first if needed. Fails (not skips) when a GPU
    is present but the library cannot be built or loaded."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from alpaca_b200 import build
    build.build()
    import alpaca_b200
    return alpaca_b200.load()

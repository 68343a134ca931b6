"""Shared pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` run on a B200 (`pytest -m gpu`); everything else runs on a
CPU-only host (`pytest -m "not gpu"`). GPU tests call the product through
libtqfsample.so and check it against the CPU oracle in oracle/.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")

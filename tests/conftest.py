"""Test configuration: the `gpu` marker, import paths, and the golden fixtures.

Tests marked `gpu` need a CUDA device and the built libekv_b200.so; every other test runs on CPU.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PACKAGE_PARENT = os.path.join(ROOT, "sigmod-kvscope_b200")
for path in (ROOT, PACKAGE_PARENT):
    if path not in sys.path:
        sys.path.insert(0, path)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libekv_b200.so")


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, f"{name}.npz"), allow_pickle=False) as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def golden():
    return load_golden


@pytest.fixture(scope="session")
def cuda_lib():
    """The built library on a CUDA device; the GPU tests fail (not skip) without one."""
    import torch

    assert torch.cuda.is_available(), "the gpu tests need a CUDA device"
    import ekv._lib as lib

    return lib.load()

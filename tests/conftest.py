"""Shared test configuration.

`-m "not gpu"` runs the oracle, host-logic and ABI-surface tests on any machine;
`-m gpu` runs the parity tests through libq38.so's C ABI on a B200.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "qwen38-mlx-swift_b200")
for p in (os.path.join(ROOT, "oracle"), PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libq38.so")


@pytest.fixture(scope="session")
def q38():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import q38 as mod  # raises if libq38.so is missing: no fallback
    return mod


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    return O

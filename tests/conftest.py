"""Shared pytest setup: the `gpu` marker, import paths and seeded inputs.

Tests marked ``gpu`` need a CUDA device (a B200) and the built extension;
everything else runs on CPU.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "qwen0.6b_b200")
for p in (PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built extension")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def weights_2l():
    from qwen_weights import synthetic_weights
    return synthetic_weights(seed=7, num_layers=2)


@pytest.fixture(scope="session")
def weights_28l():
    from qwen_weights import synthetic_weights
    return synthetic_weights(seed=1234, num_layers=28)

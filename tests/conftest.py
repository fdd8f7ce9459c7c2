"""Shared pytest configuration: the `gpu` marker, import paths, and helpers.

CPU tests (-m "not gpu") cover the oracle against the golden fixtures, the host logic and the C ABI
library (load + exports, argument checks that return before any device work).  GPU tests (-m gpu)
are the parity tests proper: the CUDA kernels, called through the C ABI / torch ops, against the
oracle on seeded inputs.
"""
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "kernel-rsi_b200"
LIBRARY = PKG / "library"
for p in (str(ROOT), str(LIBRARY)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return torch.load(ROOT / "tests" / "golden" / f"{name}_golden.pt", weights_only=True)
    return load

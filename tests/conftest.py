"""Shared test setup: import paths, the `gpu` marker, common fixtures.

Tests marked `gpu` need a CUDA device and the built libsarr.so; everything
else runs on the CPU (the oracle, the host logic, the C ABI's host-only entry
points and the gloo multi-process paths)."""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "sar-3dgs_b200")
for p in (PKG, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libsarr.so")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)

"""Shared test setup.

Markers: `gpu` tests need a CUDA device (sm_100a) and the built libkolibri_b200.so; they are
the parity tests proper and call the kernels through the C ABI.  Everything else runs on CPU.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
PKG_ROOT = REPO / "profiling-moe_b200"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def dev():
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def api():
    from kolibri_b200.api import load_api
    return load_api()

"""Shared pytest setup: the ``gpu`` marker, repo-root imports and fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
for entry in (str(ROOT), str(GOLDEN)):
    if entry not in sys.path:
        sys.path.insert(0, entry)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200) and the built kernel library")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_ops():
    return torch.load(GOLDEN / "ops.pt")


def load_golden(name: str) -> dict:
    return torch.load(GOLDEN / f"herm_{name}.pt")


@pytest.fixture
def cuda():
    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _no_device_timeouts(request):
    """After every GPU test, the library's device status word must be clear:
    a bounded device-side wait that gave up is a failure, never silent."""
    yield
    if "gpu" in request.keywords and torch.cuda.is_available():
        from koemi_5hom_b200 import _native
        if _native._LIBRARY is not None and _native._INITIALISED_DEVICES:
            for index in list(_native._INITIALISED_DEVICES):
                assert _native.device_status(torch.device("cuda", index)) == 0, "device-side wait timed out"

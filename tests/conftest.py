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

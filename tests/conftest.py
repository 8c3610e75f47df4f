"""Test configuration: import paths, the ``gpu`` marker and shared helpers."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
for p in (REPO, REPO / "cuda-learn_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN_DIR = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden_files():
    return sorted(GOLDEN_DIR.glob("*.pt"))


def load_golden(path):
    return torch.load(path, map_location="cpu", weights_only=False)

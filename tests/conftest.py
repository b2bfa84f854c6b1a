"""Shared pytest set-up.

Tests marked ``gpu`` need a CUDA device and the built library; everything else
runs on CPU (oracle against the golden fixtures, host logic, C-ABI surface).
"""
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_DIR = REPO / "event-aware-sae-trainer_b200"
for p in (REPO, PKG_DIR):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test requires a CUDA device (B200)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name):
    import numpy as np
    return dict(np.load(GOLDEN / f"{name}.npz"))

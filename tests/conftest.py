"""Shared pytest setup: the ``gpu`` marker, repo-root imports, skips.

GPU tests (``-m gpu``) need a compute-capability 10.0 device; everything else
runs on the CPU container.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "slow: large-shape GPU test")


def _have_b200() -> bool:
    try:
        import torch

        return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    except Exception:  # pragma: no cover
        return False


def pytest_collection_modifyitems(config, items):
    if _have_b200():
        return
    skip = pytest.mark.skip(reason="needs a compute capability 10.0 GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)

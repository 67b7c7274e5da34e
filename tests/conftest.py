"""Pytest configuration: the ``gpu`` marker and shared helpers.

``-m "not gpu"`` runs everywhere (oracle pinning, C-ABI symbols and shape contracts,
host logic, gloo multi-process tests). ``-m gpu`` tests need an sm_100 device; they
call the CUDA library through its C ABI and compare with the CPU oracle.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
for _p in (REPO, REPO / "tests"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _has_cuda() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


def pytest_collection_modifyitems(config, items):
    if _has_cuda():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def library():
    """The built C-ABI library (built on demand from the in-tree sources)."""
    from fast_gpu_asr_b200 import _lib
    from fast_gpu_asr_b200.build import build

    build()
    return _lib.library()

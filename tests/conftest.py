"""Shared pytest setup.

* ``gpu`` marks tests that need a CUDA device (run on a B200 with ``-m gpu``); without a
  device they are skipped.
* The package root ``radeon-kernels_b200`` and the repository root (for ``oracle``) are put
  on ``sys.path`` so ``import radeon_kernels`` and ``import oracle`` work without install.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_ROOT = REPO / "radeon-kernels_b200"
for path in (str(PKG_ROOT), str(REPO)):
    if path not in sys.path:
        sys.path.insert(0, path)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    if not any(item.get_closest_marker("gpu") for item in items):
        return
    try:
        import torch

        available = torch.cuda.is_available()
    except Exception:  # pragma: no cover - torch import failure
        available = False
    if available:
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for item in items:
        if item.get_closest_marker("gpu"):
            item.add_marker(skip)


def golden_cases(prefix: str) -> list[Path]:
    return sorted(GOLDEN.glob(f"{prefix}_*.npz"))

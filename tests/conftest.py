"""Shared test configuration.

Markers:
  gpu   needs a CUDA device (B200); run with ``-m gpu``.  Skipped when no
        device is visible.
  slow  long-running.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: requires a CUDA GPU (B200)")
    config.addinivalue_line("markers", "slow: long-running tests")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture
def seed() -> int:
    return 42


def rel_fro(x: torch.Tensor, ref: torch.Tensor) -> float:
    """||x - ref||_F / ||ref||_F in float64 (0 when both are zero)."""
    x = x.detach().double().cpu()
    ref = ref.detach().double().cpu()
    den = ref.norm().item()
    num = (x - ref).norm().item()
    if den == 0.0:
        return num
    return num / den

"""Shared test configuration.

``gpu`` tests need a CUDA device and the built ``libclef_b200.so``; everything
else runs on CPU.  The oracle under ``oracle/`` is imported only here and in
the tests, as the checker.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built CUDA library")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    """Skip ``gpu`` tests when no CUDA device is visible."""
    if not any("gpu" in item.keywords for item in items):
        return
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)

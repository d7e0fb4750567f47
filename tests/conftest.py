"""Shared pytest configuration: the ``gpu`` marker and golden-fixture access."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden.pt"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built library")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


_cases = None


def golden_cases() -> dict:
    global _cases
    if _cases is None:
        _cases = torch.load(GOLDEN, weights_only=False)
    return _cases


def golden_names(op: str) -> list[str]:
    return sorted(k for k, v in golden_cases().items() if v["op"] == op)


def rel_fro(a: torch.Tensor, b: torch.Tensor) -> float:
    """Relative Frobenius error ||a - b|| / ||b|| computed in float64."""
    a = a.detach().double().cpu()
    b = b.detach().double().cpu()
    den = torch.linalg.norm(b).item()
    num = torch.linalg.norm(a - b).item()
    return num / den if den > 0 else num

"""Shared pytest setup.

Markers:
  gpu -- needs a CUDA device and the built product library; run with ``-m gpu``.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA device (B200) and the built extension")


@pytest.fixture(scope="session", autouse=True)
def _built_checker():
    from oracle import build

    build()


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False

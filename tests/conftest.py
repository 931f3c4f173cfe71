"""Shared pytest setup: the `gpu` marker, repo import path, and the oracle build."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and the built libt2c_sm100.so")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as module

    module.build()
    return module

"""Shared test setup: the ``gpu`` marker, import paths, and the package fixture.

GPU tests (``-m gpu``) call the CUDA path through the C ABI and fail loudly if the library is missing; CPU tests
(``-m "not gpu"``) cover the oracle against the golden fixtures, the host logic and the ABI surface.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built C-ABI library")


@pytest.fixture(scope="session")
def h3b():
    import __graft_entry__
    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def ops(h3b):
    return h3b.ops

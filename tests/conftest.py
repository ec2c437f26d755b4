"""Shared test setup.

Markers
-------
gpu : needs a B200 (sm_100a).  The CPU suite runs with ``-m "not gpu"``; the
      parity tests proper run on a GPU box with ``-m gpu``.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "cuvs-silicon_b200"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a B200 GPU (sm_100a)")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle

    oracle.build_native()
    return oracle


@pytest.fixture(scope="session")
def engine():
    """The compiled engine's Python binding (the .so must exist)."""
    import cuvs_b200

    cuvs_b200.lib()
    return cuvs_b200

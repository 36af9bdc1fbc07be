"""Shared pytest setup: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs the oracle, host-logic and library-load tests on CPU;
``-m gpu`` runs the CUDA parity tests (they call through the C ABI).
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "unltd-inference_b200")
for p in (REPO, PKG, os.path.join(REPO, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def ora():
    import oracle

    oracle.lib()
    return oracle

"""Shared pytest configuration.

`gpu` marks tests that need a CUDA device (they run on a B200 box); every
other test runs on the CPU build host.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: larger CPU golden cases")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    o.build()
    return o


@pytest.fixture(scope="session")
def package_built():
    """Both shared libraries of the package, built in place (incremental)."""
    from volta_zk_b200 import build_all

    build_all()

"""Shared test setup: import paths, the `gpu` marker, oracle fixtures."""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PACKAGE_DIR = ROOT / "alpha-yoo-for-great-kingdom_b200"
for path in (str(ROOT), str(PACKAGE_DIR)):
    if path not in sys.path:
        sys.path.insert(0, path)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference
    try:
        return Reference()
    except FileNotFoundError:
        pytest.skip("the reference engine (oracle/_ref) is not built here")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        return dict(np.load(GOLDEN / name, allow_pickle=False))
    return load


def cpu_threads():
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return os.cpu_count() or 1

"""Shared fixtures.  GPU tests carry ``@pytest.mark.gpu``; everything else runs
on a CPU-only machine."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def orc():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))


@pytest.fixture(scope="session")
def ref():
    """The reference kernels compiled from source, or skip where unavailable."""
    from oracle.oracle import load_reference
    r = load_reference()
    if r is None:
        pytest.skip("reference kernels (oracle/_ref) not built or not runnable here")
    return r

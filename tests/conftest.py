"""Shared fixtures. Tests marked ``gpu`` need a B200 and the built CUDA library; everything else runs on CPU."""

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a) and the built libartlite_moe_cuda.so")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def golden():
    with np.load(os.path.join(REPO, "tests", "golden", "golden.npz")) as g:
        return {k: g[k] for k in g.files}


@pytest.fixture(scope="session")
def orc():
    from oracle import lib
    return lib.oracle()

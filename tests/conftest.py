"""Shared pytest configuration.

Markers
-------
gpu : needs a CUDA device (a B200); everything unmarked runs on the CPU.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running test")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    path = os.path.join(REPO, "tests", "golden", "glm_golden.npz")
    data = np.load(path)
    names = sorted({k.split("/")[0] for k in data.files})
    return {n: {k: data[f"{n}/{k}"] for k in ("X", "M", "Y", "yhat", "grad")} for n in names}


@pytest.fixture(scope="session")
def oracle():
    from oracle import pyoracle

    pyoracle.build()
    return pyoracle

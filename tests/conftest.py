"""Shared test setup: paths to the package, the oracle and helpers.

GPU tests carry @pytest.mark.gpu; `pytest -m "not gpu"` runs on a machine
without a GPU (oracle, golden vectors, host-side C ABI, multi-process logic)."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "dots.tts.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "slow: long CPU oracle runs")


@pytest.fixture(scope="session")
def orc():
    import oracle as O
    return O.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle as O
    if not O.Reference.available():
        pytest.skip("oracle/_ref (the reference build) is not present")
    return O.Reference()


@pytest.fixture(scope="session")
def dtts_mod():
    import dtts
    dtts.lib()
    return dtts

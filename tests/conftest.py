"""pytest configuration: the `gpu` marker and shared fixtures."""
import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def kat():
    with open(os.path.join(GOLDEN, "kat_q4_0.json")) as f:
        return json.load(f)["cases"]


@pytest.fixture(scope="session")
def projection_fixtures():
    with open(os.path.join(GOLDEN, "projection_small.json")) as f:
        return json.load(f)["cases"]


@pytest.fixture(scope="session")
def coracle():
    from oracle.q4_oracle_np import COracle
    return COracle()

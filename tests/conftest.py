"""Shared test set-up: the `gpu` marker, import paths and built libraries."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _built_libraries():
    """Build the CUDA library and the oracle once per session (no-op when current)."""
    from jlust_b200 import build as b
    b.build()
    from oracle import oracle as O
    O.build()
    yield


@pytest.fixture(scope="session")
def golden():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "kat.json")) as f:
        return json.load(f)

"""Test configuration: the `gpu` marker and import paths.

CPU tests (`-m "not gpu"`) check the oracle against the reference's own
known-answer tests, the host-side logic of the library and its exported ABI.
GPU tests (`-m gpu`) run the CUDA path through the C ABI and compare it with
the oracle on identical inputs.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("le-wm-nv_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path)")


@pytest.fixture(scope="session")
def ctx():
    import lewm_b200 as L
    c = L.Context(0)
    yield c
    c.close()

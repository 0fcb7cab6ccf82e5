"""Test configuration: the `gpu` marker and import paths for the oracle (test
infrastructure) and the product's ctypes bindings."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "hunyuan-image-3-80b.cpp_b200")
for p in (os.path.join(ROOT, "oracle"), PKG, os.path.dirname(os.path.abspath(__file__))):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (run with -m gpu)")


@pytest.fixture(scope="session")
def orc():
    import oracle as O
    return O.Oracle()

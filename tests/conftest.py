"""pytest configuration: the `gpu` marker and import paths for the package and the oracle."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "qwen-3.8-in-rust_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200); run with -m gpu")


@pytest.fixture(scope="session")
def orc():
    import oracle

    oracle.build()
    return oracle

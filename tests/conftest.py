import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200); run with -m gpu")


@pytest.fixture(scope="session")
def lib():
    from macuda_b200.cublas import library
    return library()


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle
    return oracle

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


@pytest.fixture(scope="session")
def lib():
    from tierstream_b200 import abi
    return abi.load()


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle.orc()


@pytest.fixture(scope="session")
def ref():
    import oracle
    r = oracle.ref()
    if r is None:
        pytest.skip("oracle/_ref/libtsref.so not built (the reference sources were not available)")
    return r

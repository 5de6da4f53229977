import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device; run with -m gpu")


def pytest_collection_modifyitems(config, items):
    # Keep tests/test_zz_* last even under -p randomisation plugins.
    items.sort(key=lambda it: 1 if os.path.basename(str(it.fspath)).startswith("test_zz_") else 0)


@pytest.fixture(scope="session")
def lib():
    from metalblas_b200 import _lib
    return _lib.load()

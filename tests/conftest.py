import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def native_lib():
    """The in-tree libatlas_mem.so; built here with nvcc if it is missing or stale."""
    from atlas_rnn_b200 import _lib, build
    if not build.up_to_date():
        build.build()
    return _lib.lib()

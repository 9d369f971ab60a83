import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built libmgpu.so")


@pytest.fixture(scope="session")
def dev():
    import mvlm_b200 as mg
    d = mg.Device(0)
    yield d
    d.finish()

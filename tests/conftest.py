import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")
    config.addinivalue_line("markers", "slow: takes more than ~20 s on the CPU")


def pkg(sub=None):
    name = "anima-studio_b200" + ("." + sub if sub else "")
    return importlib.import_module(name)


@pytest.fixture(scope="session")
def anima():
    return pkg()

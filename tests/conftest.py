import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "mtp-engine_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")

for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


ISOLATED_ENV = "MTP_ISOLATED_RUN"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "isolated: GPU test of a kernel awaiting its first GPU run; runs only in "
                                       "a child process started by tests/test_gpu_isolated.py")


def pytest_collection_modifyitems(config, items):
    # A fault in a kernel that has never run would leave this process's CUDA
    # context unusable for every later test; such tests run in child processes.
    if os.environ.get(ISOLATED_ENV) == "1":
        return
    skip = pytest.mark.skip(reason="runs in a child process (tests/test_gpu_isolated.py)")
    for item in items:
        if "isolated" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        return np.load(os.path.join(GOLDEN, name))

    return load

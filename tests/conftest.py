import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: runs longer than a few seconds")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def built_lib():
    """Build libqb.so once (nvcc cross-compiles without a GPU) and load it."""
    from hackthenorth_b200 import build as qbuild
    from hackthenorth_b200 import _lib

    qbuild.build()
    return _lib.load()


@pytest.fixture(scope="session")
def cpu_threads():
    import torch

    torch.set_num_threads(max(1, min(16, os.cpu_count() or 1)))
    return torch.get_num_threads()

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session", autouse=True)
def _built_library():
    """Build libgdn_b200.so when it is missing or stale (nvcc runs without a
    GPU); on a GPU box the prebuilt library that travelled with the tree is
    used as is."""
    from domesticated_torch_mlu_ops_b200 import build as b
    import shutil
    if shutil.which("nvcc") or os.path.exists("/usr/local/cuda/bin/nvcc"):
        b.build()
    yield

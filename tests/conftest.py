import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "isa-lm_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")
MODEL_CACHE = os.environ.get("KRAFLA_MODEL_DIR", os.path.join(ROOT, "_models"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and libkrafla_cuda.so")


@pytest.fixture(scope="session")
def built():
    """The C libraries this suite loads: the oracle, the model writer and the CUDA library."""
    import __graft_entry__
    __graft_entry__.build_host()
    return True

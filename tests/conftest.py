import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _oracle_built():
    from oracle import oracle as orc
    if not os.path.exists(orc.PORT_PATH):
        orc.build()


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu():
    """Skips GPU-marked tests where no GPU is present; on a GPU box the CUDA library must load."""
    if not _has_gpu():
        pytest.skip("no CUDA GPU")
    from ligguf_b200 import _lib
    return _lib.load()

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def xlib():
    from xtagger_b200 import lib as L
    return L.lib()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _release_device_buffers():
    yield
    import sys as _s
    g = _s.modules.get("tests._gpu")
    if g is not None and g._keep:
        g.release()

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a (B200) GPU")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Builds the CPU oracle and libsfb200.so once per session if stale."""
    from oracle import oracle
    from servoflow_b200 import build

    oracle.build()
    build.build_library()
    oracle.build_binding()
    yield


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu():
    if not has_gpu():
        pytest.fail("this test needs an sm_100a GPU (run with -m 'not gpu' on CPU hosts)")
    import torch
    torch.cuda.set_device(0)
    return torch.device("cuda:0")

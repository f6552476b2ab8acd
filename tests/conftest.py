import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def have_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def kl():
    import maia_b200

    maia_b200.lib()
    return maia_b200


@pytest.fixture(scope="session")
def cuda(kl):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    major, minor = torch.cuda.get_device_capability()
    assert major == 10, f"needs an sm_100 device, found sm_{major}{minor}"
    kl.set_wait_timeout_ns(1_000_000_000)
    return torch.device("cuda:0")

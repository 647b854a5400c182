import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: full-size parity cases (seconds of CPU oracle work)")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100, found sm_{major}{minor}")
    # the product path has no fallback: the native library must be there
    from ratchet_b200 import _lib

    _lib.lib()
    return torch.device("cuda:0")


def pytest_collection_modifyitems(config, items):
    # keep a stable order: CPU tests first, then GPU tests in file order
    pass

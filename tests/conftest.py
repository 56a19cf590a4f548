import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is not available")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail(f"GPU tests need an sm_100 device, found sm_{major}x")
    return torch.device("cuda", 0)

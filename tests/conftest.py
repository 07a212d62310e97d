import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        pytest.fail(f"kernels are built for sm_100a only, device is sm_{major}{minor}")
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return np.load(os.path.join(REPO, "tests", "golden", "awq_reference_golden.npz"))

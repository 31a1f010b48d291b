import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; runs the CUDA rows against the CPU oracle")


@pytest.fixture(scope="session")
def oracle_lib():
    import harness
    return harness.oracle()


@pytest.fixture(scope="session")
def product_lib():
    import harness
    return harness.product()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device visible")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"device 0 is sm_{major}{minor}; this library is built for sm_100a only")
    return torch

import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    return importlib.import_module("truellm-engine_b200")


@pytest.fixture(scope="session")
def ops(pkg):
    return importlib.import_module("truellm-engine_b200.ops")


@pytest.fixture(scope="session")
def wl(pkg):
    return importlib.import_module("truellm-engine_b200.workloads")


@pytest.fixture(scope="session")
def O():
    from oracle import oracle as mod
    mod.build()
    return mod


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda:0")

import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built CUDA library")


@pytest.fixture(scope="session")
def ge():
    """The product package (gemma-embed-swift_b200)."""
    return importlib.import_module("gemma-embed-swift_b200")


@pytest.fixture(scope="session")
def synth():
    return importlib.import_module("gemma-embed-swift_b200.synthetic")


@pytest.fixture(scope="session")
def oracle():
    from oracle import binding
    binding.lib()
    return binding


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device; run them on a B200 box")
    major, _ = torch.cuda.get_device_capability(0)
    assert major == 10, "GPU tests need an sm_100 (B200) device"
    return 0


@pytest.fixture(scope="session")
def cuda_available():
    import torch
    return torch.cuda.is_available()

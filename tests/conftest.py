import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built CUDA extension")


def gpu_available() -> bool:
    import torch
    if not torch.cuda.is_available():
        return False
    major, _ = torch.cuda.get_device_capability(0)
    return major == 10


@pytest.fixture(scope="session")
def attn():
    """The product module; a GPU test fails loudly (no skip) when the native
    extension is missing on a GPU box."""
    import rocm_attn_b200
    return rocm_attn_b200

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    assert torch.cuda.is_available(), "GPU test collected on a machine without CUDA"
    from smat_attention_b200 import _lib
    _lib.check("smat_device_supported", _lib.lib().smat_device_supported(0))
    return torch.device("cuda", 0)

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "gtx16-fp16_b200")
for p in (ROOT, PKG_ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built libg16.so")


@pytest.fixture(scope="session")
def cuda_ok():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True

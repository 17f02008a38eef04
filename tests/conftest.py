import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

# The reference source tree (read-only); only CPU tests that cross-check the
# oracle live against it use this, and they skip when it is absent.
REFERENCE_ROOT = os.environ.get("LOOPSPEC_REFERENCE", "/root/reference")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA extension")


def reference_available():
    return os.path.isdir(os.path.join(REFERENCE_ROOT, "sglang_recurrent", "loopspec"))


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    return torch.device("cuda:0")

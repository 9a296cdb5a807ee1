import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (runs on the B200 box)")


@pytest.fixture(scope="session")
def kat():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "kat.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def cuda():
    """torch with a visible CUDA device (for device buffers only)."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test collected without a CUDA device")
    torch.cuda.init()
    return torch

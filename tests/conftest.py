import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

REFERENCE_DIRS = [os.path.join(ROOT, "baseline", "_ref")]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    config.addinivalue_line("markers", "reference: needs the reference package as an oracle")
    config.addinivalue_line("markers", "slow: slower CPU test")


def reference_available() -> bool:
    return any(os.path.isdir(os.path.join(d, "src")) for d in REFERENCE_DIRS)


def import_reference():
    for d in REFERENCE_DIRS:
        if os.path.isdir(os.path.join(d, "src")) and d not in sys.path:
            sys.path.insert(0, d)


@pytest.fixture
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (compute capability 10.0) GPU")


def _has_b200() -> bool:
    try:
        import torch
    except Exception:
        return False
    return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)


HAS_B200 = _has_b200()


def pytest_collection_modifyitems(config, items):
    if HAS_B200:
        return
    skip = pytest.mark.skip(reason="needs a B200 GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) CUDA device")
    config.addinivalue_line("markers", "slow: long-running")


def _has_b200():
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    run_slow = os.environ.get("FFB_SLOW") == "1"
    has_gpu = _has_b200()
    skip_gpu = pytest.mark.skip(reason="no B200 (sm_100a) device visible")
    skip_slow = pytest.mark.skip(reason="long-running; set FFB_SLOW=1")
    for item in items:
        if "gpu" in item.keywords and not has_gpu:
            item.add_marker(skip_gpu)
        elif "slow" in item.keywords and not run_slow:
            item.add_marker(skip_slow)

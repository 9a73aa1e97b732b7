import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
PACKAGE_ROOT = ROOT / "sm120-norm-fusion-kernels_b200"
for path in (str(ROOT), str(PACKAGE_ROOT), str(ROOT / "tests")):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    # GPU tests only skip where there is no GPU at all; on a GPU host a missing
    # extension makes them fail loudly.
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)

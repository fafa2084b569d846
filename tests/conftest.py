"""Test configuration: registers the `gpu` marker and puts the package and the
oracle on sys.path. GPU tests run with device-side error checks enabled."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "fast-mac-gsplat_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))
os.environ.setdefault("GSPLAT_B200_CHECK", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)

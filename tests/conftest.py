"""Test configuration: the `gpu` marker and shared helpers.

`-m "not gpu"` runs on any machine (oracle vs golden fixtures, host logic,
library load / exports, gloo SPMD). `-m gpu` needs a B200 and runs the
kernels through the C ABI against the oracle.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

# Kernel waits in tests give up after 10 s rather than the 4 s default x many.
os.environ.setdefault("TRNBLAS_B200_WAIT_NS", "10000000000")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")


def has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)

"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on a CPU-only machine: the oracle against the reference's golden
fixtures, host-side logic, the C-ABI library's exports and the gloo multi-rank schedule.
`-m gpu` runs on a B200: the CUDA kernels against the oracle through the C-ABI.
"""

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
for p in (REPO, REPO / "mlx-primitives_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")
    config.addinivalue_line("markers", "slow: long-running test")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)

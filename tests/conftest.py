"""pytest configuration: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs on a host without a GPU (oracle, golden fixtures, C-ABI
exports and argument checks, host logic, gloo multi-rank tests);
``-m gpu`` runs the parity tests through the C-ABI on a B200.
"""

from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "flash-kmeans-cuda_b200")
for p in (PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the CUDA kernels")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    return torch.device("cuda", 0)

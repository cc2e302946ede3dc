"""Shared pytest configuration.

``-m gpu`` tests need a CUDA device and the in-tree ``libmxfa_b200.so``;
everything else runs on the CPU (the driver runs ``-m "not gpu"`` without a
GPU).
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN_DIR = os.path.join(REPO, "tests", "golden")
for path in (REPO, GOLDEN_DIR):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    with np.load(os.path.join(GOLDEN_DIR, "golden.npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but torch.cuda.is_available() is False")
    return torch.device("cuda", 0)

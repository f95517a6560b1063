"""pytest configuration: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs the oracle, golden-vector, ABI and host-logic tests on
any machine; ``-m gpu`` runs the CUDA parity tests (B200 required).
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "macqwen-releases_b200"
for p in (str(ROOT), str(PKG_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    with np.load(GOLDEN / "reference_numpy.npz") as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def cuda_lib():
    """The loaded library after device initialisation (GPU tests only)."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test ran without a CUDA device")
    from flashnext_b200 import _lib

    return _lib.ensure_device()

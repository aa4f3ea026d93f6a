"""Test configuration: package path, the ``gpu`` marker and shared helpers.

``-m "not gpu"`` runs everything that needs no GPU (oracle pinning, C-ABI
exports, host logic, gloo multi-process logic); ``-m gpu`` runs the parity
tests on a B200. GPU tests do not skip when CUDA is missing: they fail.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "llm-tensorcore-hgemm_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN / "hgemm_golden.npz") as data:
        return {k: data[k] for k in data.files}

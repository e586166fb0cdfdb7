import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through libmatrixman_b200 on cuda:0)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(GOLDEN / "reference_vectors.npz"))


@pytest.fixture(scope="session")
def mm():
    """The product package with the device runtime initialised (GPU tests only)."""
    import matrixman_b200 as matrixman
    matrixman.init()
    return matrixman

"""Shared test setup: import paths for the package and the oracle, the `gpu` marker."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "useful-work-coin_b200")
for p in (ROOT, PKG_ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    import json

    import numpy as np
    with open(os.path.join(GOLDEN, "golden.json")) as f:
        meta = json.load(f)
    arrays = dict(np.load(os.path.join(GOLDEN, "golden.npz")))
    return meta, arrays


@pytest.fixture(scope="session")
def dev():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def det_golden():
    """Vectors from the reference's detrt (tests/golden/make_golden_det.py)."""
    import numpy as np
    return dict(np.load(os.path.join(GOLDEN, "det_golden.npz")))

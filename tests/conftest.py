import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "sage_golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and libsage_sm100.so")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


class Golden:
    """Fixture cases from tests/golden/sage_golden.npz (made by tests/golden/make_golden.py)."""

    def __init__(self, path):
        self.z = np.load(path)
        self.cases = sorted({k.split("/")[0] for k in self.z.files})

    def __call__(self, case, key):
        return self.z[f"{case}/{key}"]

    def has(self, case, key):
        return f"{case}/{key}" in self.z.files


@pytest.fixture(scope="session")
def golden():
    return Golden(GOLDEN)

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN_DIR = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


class Golden:
    """Accessor for tests/golden/golden.npz (+ golden.json)."""

    def __init__(self):
        import json

        self.arrays = np.load(os.path.join(GOLDEN_DIR, "golden.npz"))
        with open(os.path.join(GOLDEN_DIR, "golden.json")) as f:
            self.meta = json.load(f)

    def __getitem__(self, k):
        return self.arrays[k]

    def csr(self, prefix):
        """Return oracle.CSR built from stored arrays with this prefix."""
        from oracle import oracle as O

        a = self.arrays
        M, K = (int(v) for v in a[prefix + "shape"])
        return O.CSR(M, K, a[prefix + "values"].copy(), a[prefix + "cols"].copy(),
                     a[prefix + "row_start"].copy(), a[prefix + "row_nnz"].copy(),
                     a[prefix + "row_capacity"].copy())


@pytest.fixture(scope="session")
def golden():
    return Golden()

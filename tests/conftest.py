"""Shared fixtures: the golden-fixture loader, GPU gating and the oracle.

Tests marked ``gpu`` need a CUDA device and the built libpiton_b200.so; the
rest run on CPU.  The oracle (``oracle/``) is the checker of the GPU tests and
is itself pinned against the reference emulator's golden outputs.
"""

import glob
import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (CUDA) device and libpiton_b200.so")


class Golden:
    def __init__(self, path):
        self.path = path
        self.name = os.path.splitext(os.path.basename(path))[0]
        z = np.load(path)
        self.meta = json.loads(str(z["meta"]))
        self.arrays = {k: z[k] for k in z.files if k != "meta"}

    def __getitem__(self, k):
        return self.arrays[k]

    def __contains__(self, k):
        return k in self.arrays

    def __repr__(self):
        return self.name


def goldens(prefix: str):
    return [Golden(p) for p in sorted(glob.glob(os.path.join(GOLDEN, prefix + "*.npz")))]


def golden_ids(gs):
    return [g.name for g in gs]


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def sha256(a: np.ndarray) -> str:
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def max_ulp(a, b):
    """Largest distance in float32 units in the last place (same-sign finite values)."""
    ai = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    bi = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFFFFFF), bi)
    return int(np.abs(ai - bi).max()) if ai.size else 0


def dot_error(c, ref):
    """Normalised dot-product error max|c - ref| / max|ref| (the reference's
    'normalized error', piton/runtime/pi.py:470-528)."""
    ref = np.asarray(ref, np.float64)
    return float(np.abs(np.asarray(c, np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))

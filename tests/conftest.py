"""Shared fixtures: import paths, the `gpu` marker, seeded RNG, the reference's
rel_err metric (tests/conftest.py:15-18 in Nags-gk/nki-kernel-lab) and golden loading."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "nki-kernel-lab_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built library")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture
def rng():
    return np.random.default_rng(1234)


def rel_err(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-12))


def load_golden(name: str) -> dict:
    """npz -> {key: array}; keys stored as '<key>@bf16' come back as ml_dtypes.bfloat16."""
    import ml_dtypes

    out = {}
    with np.load(os.path.join(GOLDEN, name)) as z:
        for k in z.files:
            if k.endswith("@bf16"):
                out[k[:-5]] = z[k].view(ml_dtypes.bfloat16)
            else:
                out[k] = z[k]
    return out


def cases(golden: dict) -> list[str]:
    return sorted({k.split("/")[0] for k in golden})


def to_torch(a):
    """NumPy (float32 / ml_dtypes.bfloat16) -> CPU torch tensor of the same dtype."""
    import ml_dtypes
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == ml_dtypes.bfloat16:
        return torch.from_numpy(a.view(np.uint16).copy()).view(torch.bfloat16)
    return torch.from_numpy(a.copy())


def to_numpy(t):
    import ml_dtypes
    import torch

    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.uint16).numpy().view(ml_dtypes.bfloat16)
    return t.numpy()


def bf16_ulp_diff(a, b) -> np.ndarray:
    """Distance in bf16 ulps between two bf16 arrays (monotone integer mapping)."""
    def key(x):
        u = np.asarray(x).view(np.uint16).astype(np.int32)
        return np.where(u & 0x8000, 0x8000 - (u & 0x7FFF), 0x8000 + u)
    return np.abs(key(a) - key(b))

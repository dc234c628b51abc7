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


def bf16_spacing(v) -> np.ndarray:
    """Gap between adjacent bf16 values at |v| (one ulp), elementwise."""
    a = np.abs(np.asarray(v, dtype=np.float32))
    return np.exp2(np.floor(np.log2(np.maximum(a, np.float32(2.0 ** -126)))) - 7)


def bf16_excess_rel(a, b) -> float:
    """rel_err after allowing each element one bf16 ulp for the final output rounding:
    max(|a - b| - ulp(b), 0) / max|b|. Two correct bf16 pipelines that differ only in
    fp32 accumulation order can disagree by one output ulp anywhere, which alone can
    exceed a 3e-3 plain rel_err when |b| reaches 4; this metric measures the error the
    computation adds beyond that unavoidable rounding."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    return float(np.maximum(np.abs(a - b) - bf16_spacing(b), 0).max() / max(np.abs(b).max(), 1e-12))

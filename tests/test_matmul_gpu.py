"""GPU parity of the GEMM kernels (tcgen05 bf16, exact fp32, naive)."""
from __future__ import annotations

import ml_dtypes
import numpy as np
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from conftest import bf16_excess_rel, bf16_ulp_diff, cases, load_golden, rel_err, to_numpy, to_torch
from oracle import nki_oracle as O

pytestmark = pytest.mark.gpu
BF16 = ml_dtypes.bfloat16
MM = load_golden("golden_matmul.npz")


@pytest.fixture(scope="module")
def ops():
    from nkilab import ops as _ops

    return _ops


def check_bf16(out, ref, rel=1e-2):
    """BASELINE bf16 GEMM tolerance (rel_err < 1e-2) plus a tighter sanity bound: beyond
    one ulp for the output rounding, no element is off by more than 2^-8 of max|ref|
    (a CPU fp32-vs-fp64 accumulation comparison of the same products stays near
    0.3 * 2^-8)."""
    assert out.dtype == BF16 and out.shape == ref.shape
    o, r = out.astype(np.float32), ref.astype(np.float32)
    err = rel_err(o, r)
    exc = bf16_excess_rel(o, r)
    d = bf16_ulp_diff(out, ref)
    diag = f"rel_err={err:.3e} excess={exc:.3e} ulp>1 frac={(d > 1).mean():.2e}"
    assert err < rel, diag
    assert exc < 2.0 ** -8, diag


@pytest.mark.parametrize("case", cases(MM))
@pytest.mark.parametrize("variant", ["blocked", "naive"])
def test_matmul_matches_reference_golden(ops, case, variant):
    a, b = MM[f"{case}/a"], MM[f"{case}/b"]
    out = ops.matmul(a, b, variant=variant)
    gold = MM[f"{case}/out_{variant}"]
    if gold.dtype == BF16:
        check_bf16(out, gold)
    else:
        assert out.dtype == np.float32 and rel_err(out, gold) < 1e-5


@pytest.mark.parametrize("variant", ["naive", "blocked"])
@pytest.mark.parametrize("M,K,N", [(128, 128, 512), (256, 384, 1024), (200, 300, 130), (1, 7, 3)])
def test_matmul_fp32(ops, rng, variant, M, K, N):
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((K, N)).astype(np.float32)
    assert rel_err(ops.matmul(a, b, variant=variant), a @ b) < 1e-5


@pytest.mark.parametrize("variant", ["naive", "blocked"])
def test_matmul_bf16_accumulates_in_fp32(ops, rng, variant):
    a = rng.standard_normal((256, 1024)).astype(BF16)
    b = rng.standard_normal((1024, 1024)).astype(BF16)
    ref = a.astype(np.float32) @ b.astype(np.float32)
    out = ops.matmul(a, b, variant=variant)
    assert out.dtype == BF16
    assert rel_err(out, ref) < 1e-2


@settings(max_examples=12, deadline=None)
@given(M=st.integers(1, 300), K=st.integers(1, 300), N=st.integers(1, 700))
def test_matmul_property_any_shape(M, K, N):
    from nkilab import ops

    rng = np.random.default_rng(M * 1000003 + K * 1009 + N)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    out = ops.matmul(a, b)
    assert out.shape == (M, N)
    np.testing.assert_allclose(out, a @ b, rtol=1e-4, atol=1e-4)


@settings(max_examples=16, deadline=None)
@given(M=st.integers(1, 700), K=st.integers(1, 600), N=st.integers(1, 700))
def test_matmul_bf16_property_any_shape(M, K, N):
    """Any shape through the tensor-core path (partial tiles, K/N padding)."""
    from nkilab import ops

    g = torch.Generator().manual_seed(M * 7919 + K * 31 + N)
    a = (torch.rand(M, K, generator=g) * 2 - 1).to(torch.bfloat16)
    b = (torch.rand(K, N, generator=g) * 2 - 1).to(torch.bfloat16)
    out = ops.matmul(a.cuda(), b.cuda())
    check_bf16(to_numpy(out), to_numpy(O.matmul(a, b)))


@pytest.mark.parametrize("M,K,N", [(128, 64, 128), (129, 72, 264), (1, 8, 8), (300, 1000, 520), (1024, 1024, 1024),
                                   (2048, 512, 4096)])
def test_matmul_bf16_tiles(ops, M, K, N):
    g = torch.Generator().manual_seed(M + K + N)
    a = (torch.rand(M, K, generator=g) * 2 - 1).to(torch.bfloat16)
    b = (torch.rand(K, N, generator=g) * 2 - 1).to(torch.bfloat16)
    out = ops.matmul(a.cuda(), b.cuda())
    check_bf16(to_numpy(out), to_numpy(O.matmul(a, b)))


def test_matmul_8192_cube_sampled_rows(ops):
    """BASELINE's large config: full product on the GPU, 96 random rows checked on the CPU."""
    g = torch.Generator().manual_seed(8192)
    a = (torch.rand(8192, 8192, generator=g) * 2 - 1).to(torch.bfloat16)
    b = (torch.rand(8192, 8192, generator=g) * 2 - 1).to(torch.bfloat16)
    out = ops.matmul(a.cuda(), b.cuda()).cpu()
    rows = torch.randperm(8192, generator=g)[:96]
    ref = O.matmul(a[rows], b)
    check_bf16(to_numpy(out[rows]), to_numpy(ref))


def test_kernel_level_blocked_and_naive(rng):
    from nkilab.kernels import matmul as mm

    lhsT = rng.standard_normal((256, 256)).astype(np.float32)
    rhs = rng.standard_normal((256, 1024)).astype(np.float32)
    ref = lhsT.T @ rhs
    assert rel_err(mm.matmul_blocked(lhsT, rhs, BM=2, BN=2), ref) < 1e-5
    assert rel_err(mm.matmul_naive(lhsT, rhs), ref) < 1e-5

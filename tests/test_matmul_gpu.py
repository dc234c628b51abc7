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
                                   (2048, 512, 4096), (4000, 1000, 3000)])
def test_matmul_bf16_tiles(ops, M, K, N):
    """Every tile width (64, 128, 256 columns), the last case with partial tiles in M, N and K."""
    g = torch.Generator().manual_seed(M + K + N)
    a = (torch.rand(M, K, generator=g) * 2 - 1).to(torch.bfloat16)
    b = (torch.rand(K, N, generator=g) * 2 - 1).to(torch.bfloat16)
    out = ops.matmul(a.cuda(), b.cuda())
    check_bf16(to_numpy(out), to_numpy(O.matmul(a, b)))


@pytest.mark.parametrize("M,K,N", [(4096, 4096, 4096), (4000, 1000, 3000)])
def test_matmul_replayed_from_a_graph_on_a_side_stream(ops, M, K, N):
    """Large GEMMs captured into a CUDA graph on a non-default stream, where programmatic
    dependent launch takes effect between consecutive launches: the replays give the eager
    results bit for bit and leave no device-side error."""
    from nkilab import _native as N_

    g = torch.Generator(device="cuda").manual_seed(M + N)
    a = (torch.rand(M, K, device="cuda", generator=g) * 2 - 1).to(torch.bfloat16)
    b = (torch.rand(K, N, device="cuda", generator=g) * 2 - 1).to(torch.bfloat16)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        eager = [torch.ops.nkilab.matmul(a, b, False) for _ in range(3)]
    torch.cuda.synchronize()
    N_.check_device(s.cuda_stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            replayed = [torch.ops.nkilab.matmul(a, b, False) for _ in range(3)]
    for _ in range(2):
        with torch.cuda.stream(s):
            graph.replay()
        torch.cuda.synchronize()
        N_.check_device(s.cuda_stream)
        assert all(torch.equal(r, eager[0]) for r in replayed)
    assert all(torch.equal(e, eager[0]) for e in eager)
    check_bf16(to_numpy(eager[0][:256].cpu()), to_numpy(O.matmul(a[:256].cpu(), b.cpu())))
    del graph


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


@pytest.mark.parametrize("M,K,F", [(128, 64, 128), (300, 1000, 256), (1024, 4096, 1024), (4096, 512, 11008)])
def test_matmul_swiglu_fused_equals_unfused(ops, M, K, F):
    """One GEMM over the interleaved [gate | up] weight with SwiGLU in its epilogue gives
    the same bf16 result as matmul -> matmul -> swiglu (both round gate and up to bf16
    before silu(gate) * up), and matches the oracle's unfused path within 1e-2."""
    from nkilab import _torch_ops

    g = torch.Generator().manual_seed(M + K + F)
    a = (torch.rand(M, K, generator=g) * 2 - 1).to(torch.bfloat16).cuda()
    wg = (torch.randn(K, F, generator=g) * 0.05).to(torch.bfloat16).cuda()
    wu = (torch.randn(K, F, generator=g) * 0.05).to(torch.bfloat16).cuda()
    fused = torch.ops.nkilab.matmul_swiglu(a, _torch_ops.interleave_gate_up(wg, wu))
    unfused = ops.swiglu(ops.matmul(a, wg), ops.matmul(a, wu))
    assert fused.shape == (M, F)
    assert torch.equal(fused, unfused)
    rows = torch.arange(0, M, max(1, M // 64))
    ref = O.swiglu(O.matmul(a[rows].cpu(), wg.cpu()), O.matmul(a[rows].cpu(), wu.cpu()))
    check_bf16(to_numpy(fused[rows].cpu()), to_numpy(ref))


def test_matmul_swiglu_rejects_bad_shapes(ops):
    from nkilab import _native as N

    a = torch.zeros(128, 64, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(64, 2 * 100, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(128, 100, dtype=torch.bfloat16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = N.lib.nkl_matmul_swiglu(a.data_ptr(), b.data_ptr(), out.data_ptr(), 128, 100, 64, N.BFLOAT16, st)
    assert rc == N.ERR_SHAPE and "F % 128" in N.lib.nkl_last_error().decode()
    rc = N.lib.nkl_matmul_swiglu(a.data_ptr(), b.data_ptr(), out.data_ptr(), 128, 128, 64, N.FLOAT32, st)
    assert rc == N.ERR_DTYPE


@pytest.mark.parametrize("M,N,K", [(256, 512, 384), (4096, 4096, 11008), (1000, 264, 72), (3, 8, 8)])
def test_matmul_residual_equals_matmul_then_add(M, N, K):
    """The residual add folded into the GEMM epilogue gives the same bits as a bf16 matmul
    followed by a bf16 add (the product is rounded to bf16 before the add)."""
    from nkilab import ops

    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = (torch.rand(M, K, device="cuda", generator=g) * 2 - 1).to(torch.bfloat16)
    b = (torch.rand(K, N, device="cuda", generator=g) * 2 - 1).to(torch.bfloat16)
    r = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16)
    got = torch.ops.nkilab.matmul_residual(a, b, r)
    ref = r + ops.matmul(a, b)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)

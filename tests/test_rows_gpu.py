"""GPU parity of the row kernels (RMSNorm, softmax fused / unfused, SwiGLU).

Checks the CUDA path (nkilab.ops -> torch.ops.nkilab -> C ABI) against the golden
vectors from the reference's kernels, against the CPU oracle at the BASELINE sizes,
and against the reference tests' PyTorch references and tolerances."""
from __future__ import annotations

import ctypes

import ml_dtypes
import numpy as np
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from conftest import bf16_ulp_diff, cases, load_golden, rel_err, to_numpy, to_torch
from oracle import nki_oracle as O

pytestmark = pytest.mark.gpu
BF16 = ml_dtypes.bfloat16
NORM = load_golden("golden_norm.npz")


@pytest.fixture(scope="module")
def ops():
    from nkilab import ops as _ops

    return _ops


def check_close(out, ref, fp32_rel=1e-5, bf16_rel=1e-2):
    assert out.shape == ref.shape and out.dtype == ref.dtype
    if ref.dtype == BF16:
        assert rel_err(out.astype(np.float32), ref.astype(np.float32)) < bf16_rel
        d = bf16_ulp_diff(out, ref)
        assert d.max() <= 2, f"max ulp diff {d.max()}"
    else:
        assert rel_err(out, ref) < fp32_rel


# ------------------------------------------------------------------ golden vectors

@pytest.mark.parametrize("case", [c for c in cases(NORM) if c.startswith("softmax")])
def test_softmax_matches_reference_golden(ops, case):
    x = NORM[f"{case}/x"]
    check_close(ops.softmax(x, fused=True), NORM[f"{case}/out_fused"])
    check_close(ops.softmax(x, fused=False), NORM[f"{case}/out_unfused"])


@pytest.mark.parametrize("case", [c for c in cases(NORM) if c.startswith("rmsnorm")])
def test_rmsnorm_matches_reference_golden(ops, case):
    check_close(ops.rmsnorm(NORM[f"{case}/x"], NORM[f"{case}/w"]), NORM[f"{case}/out"])


@pytest.mark.parametrize("case", [c for c in cases(NORM) if c.startswith("swiglu")])
def test_swiglu_matches_reference_golden(ops, case):
    check_close(ops.swiglu(NORM[f"{case}/gate"], NORM[f"{case}/up"]), NORM[f"{case}/out"])


# ------------------------------------------------------------------ BASELINE configs vs oracle

def _baseline_inputs(seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(4096, 2048, generator=g).to(torch.bfloat16)
    gamma = (1.0 + 0.1 * torch.randn(2048, generator=g)).to(torch.bfloat16)
    up = torch.randn(4096, 2048, generator=g).to(torch.bfloat16)
    return x, gamma, up


def test_rmsnorm_baseline_config(ops):
    x, gamma, _ = _baseline_inputs()
    out = ops.rmsnorm(x.cuda(), gamma.cuda(), 1e-6)
    check_close(to_numpy(out), to_numpy(O.rmsnorm(x, gamma, 1e-6)))


def test_softmax_baseline_config(ops):
    x, _, _ = _baseline_inputs(1)
    out = ops.softmax(x.cuda())
    ref = to_numpy(O.softmax_fused(x))
    check_close(to_numpy(out), ref)
    np.testing.assert_allclose(to_numpy(out).astype(np.float32).sum(-1), 1.0, atol=2e-2)


def test_swiglu_baseline_config(ops):
    g, _, u = _baseline_inputs(2)
    out = ops.swiglu(g.cuda(), u.cuda())
    check_close(to_numpy(out), to_numpy(O.swiglu(g, u)))


# ------------------------------------------------------------------ reference tests' checks

@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("R,D", [(128, 64), (1000, 2048), (5, 3)])
def test_softmax_matches_torch(ops, rng, fused, R, D):
    x = (rng.standard_normal((R, D)) * 4).astype(np.float32)
    out = ops.softmax(x, fused=fused)
    np.testing.assert_allclose(out, torch.softmax(torch.from_numpy(x), -1).numpy(), rtol=1e-5, atol=1e-6)


def test_softmax_is_stable_for_large_logits(ops, rng):
    x = (rng.standard_normal((256, 512)) * 1e4).astype(np.float32)
    out = ops.softmax(x)
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out.sum(-1), 1.0, atol=1e-5)


@settings(max_examples=10, deadline=None)
@given(R=st.integers(1, 400), D=st.integers(1, 1024), s=st.floats(0.1, 50))
def test_softmax_property_rows_sum_to_one(R, D, s):
    from nkilab import ops

    x = (np.random.default_rng(R * 7 + D).standard_normal((R, D)) * s).astype(np.float32)
    out = ops.softmax(x)
    np.testing.assert_allclose(out.sum(-1), 1.0, atol=1e-5)
    assert (out >= 0).all()


@pytest.mark.parametrize("R,D", [(128, 256), (300, 1024), (7, 33)])
def test_rmsnorm_matches_torch(ops, rng, R, D):
    x = rng.standard_normal((R, D)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, D).astype(np.float32)
    xt = torch.from_numpy(x)
    ref = (xt * torch.rsqrt(xt.pow(2).mean(-1, keepdim=True) + 1e-6) * torch.from_numpy(w)).numpy()
    assert rel_err(ops.rmsnorm(x, w), ref) < 1e-5


def test_rmsnorm_bf16(ops, rng):
    x = rng.standard_normal((256, 512)).astype(BF16)
    w = np.ones(512, BF16)
    xf = x.astype(np.float32)
    ref = xf / np.sqrt((xf ** 2).mean(-1, keepdims=True) + 1e-6)
    assert rel_err(ops.rmsnorm(x, w).astype(np.float32), ref) < 1e-2


def test_swiglu_matches_torch(ops, rng):
    g = rng.standard_normal((300, 1024)).astype(np.float32)
    u = rng.standard_normal((300, 1024)).astype(np.float32)
    ref = (torch.nn.functional.silu(torch.from_numpy(g)) * torch.from_numpy(u)).numpy()
    assert rel_err(ops.swiglu(g, u), ref) < 1e-5


# ------------------------------------------------------------------ edge cases

@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("R,D", [(1, 1), (3, 7), (17, 1001), (2, 8192), (9, 5000), (33, 4096), (1, 8)])
def test_row_kernels_any_shape(ops, dtype, R, D):
    g = torch.Generator().manual_seed(R * 131 + D)
    x = torch.randn(R, D, generator=g).to(dtype)
    w = torch.rand(D, generator=g).add(0.5).to(dtype)
    u = torch.randn(R, D, generator=g).to(dtype)
    xd, wd, ud = x.cuda(), w.cuda(), u.cuda()
    tol = dict(fp32_rel=2e-5, bf16_rel=1e-2)
    check_close(to_numpy(ops.rmsnorm(xd, wd)), to_numpy(O.rmsnorm(x, w)), **tol)
    check_close(to_numpy(ops.softmax(xd, True)), to_numpy(O.softmax_fused(x)), **tol)
    check_close(to_numpy(ops.softmax(xd, False)), to_numpy(O.softmax_unfused(x)), **tol)
    check_close(to_numpy(ops.swiglu(xd, ud)), to_numpy(O.swiglu(x, u)), **tol)


def test_row_kernels_unaligned_views(ops):
    """Rows starting off a 16-byte boundary take the scalar path and stay exact."""
    base = torch.randn(65 * 64 + 1, dtype=torch.float32).to(torch.bfloat16).cuda()
    x = base[1:].view(65, 64)  # 2-byte offset
    assert x.data_ptr() % 16 != 0
    w = torch.ones(64, dtype=torch.bfloat16, device="cuda")
    check_close(to_numpy(ops.rmsnorm(x, w)), to_numpy(O.rmsnorm(x.cpu(), w.cpu())))
    check_close(to_numpy(ops.softmax(x)), to_numpy(O.softmax_fused(x.cpu())))


def test_empty_rows(ops):
    x = torch.empty(0, 64, device="cuda", dtype=torch.bfloat16)
    assert ops.softmax(x).shape == (0, 64)
    assert ops.swiglu(x, x).shape == (0, 64)


def test_c_abi_direct_call():
    """Call the exported C entry point with raw device pointers (the FFI a host
    language would bind), then check the device-failure flag."""
    from nkilab import _native as N

    g = torch.Generator().manual_seed(3)
    x = torch.randn(64, 2048, generator=g).to(torch.bfloat16)
    w = torch.ones(2048, dtype=torch.bfloat16)
    xd, wd = x.cuda(), w.cuda()
    y = torch.empty_like(xd)
    st = torch.cuda.current_stream().cuda_stream
    rc = N.lib.nkl_rmsnorm(ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(wd.data_ptr()),
                           ctypes.c_void_p(y.data_ptr()), 64, 2048, 1e-6, N.BFLOAT16, ctypes.c_void_p(st))
    assert rc == N.OK
    N.check_device(st)
    check_close(to_numpy(y), to_numpy(O.rmsnorm(x, w)))


def _rope_reference(x: torch.Tensor, base: float, pos_offset: int) -> torch.Tensor:
    """Rotate-half rotary embedding in fp64 (the Llama / Hugging Face formulation)."""
    H, S, d = x.shape
    inv_freq = 1.0 / (base ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    ang = (torch.arange(S, dtype=torch.float64) + pos_offset)[:, None] * inv_freq[None, :]
    cos, sin = torch.cos(ang), torch.sin(ang)
    x1, x2 = x[..., : d // 2].double(), x[..., d // 2:].double()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1)


@pytest.mark.parametrize("H,S,d,dt,base,off", [(8, 2048, 128, torch.bfloat16, 10000.0, 0),
                                               (2, 300, 64, torch.float32, 10000.0, 0),
                                               (4, 129, 128, torch.float32, 500000.0, 4000),
                                               (1, 17, 16, torch.bfloat16, 10000.0, 7)])
def test_rope_matches_fp64_reference(H, S, d, dt, base, off):
    from nkilab import ops

    g = torch.Generator().manual_seed(H + S + d)
    x = torch.randn(H, S, d, generator=g).to(dt)
    got = ops.rope(x.cuda(), base, off).cpu()
    ref = _rope_reference(x, base, off)
    err = (got.double() - ref).abs().max().item()
    if dt == torch.float32:
        # fp32 angle = pos * theta carries ~pos * 2^-24 rad of rounding, as in any fp32 RoPE
        assert err < 1e-5 + (S + off) * 2.0 ** -22
    else:
        assert err / ref.abs().max().item() < 1e-2


def test_rope_in_place_and_bad_shapes():
    from nkilab import _native as N

    x = torch.randn(2, 64, 128, device="cuda").to(torch.bfloat16)
    want = torch.ops.nkilab.rope(x, 10000.0, 0)
    st = torch.cuda.current_stream().cuda_stream
    assert N.lib.nkl_rope(x.data_ptr(), x.data_ptr(), 2, 64, 128, 10000.0, 0, N.BFLOAT16, st) == N.OK
    assert torch.equal(x, want)
    assert N.lib.nkl_rope(x.data_ptr(), x.data_ptr(), 2, 64, 120, 10000.0, 0, N.BFLOAT16, st) == N.ERR_SHAPE
    assert N.lib.nkl_rope(x.data_ptr(), x.data_ptr(), 2, 64, 128, 1.0, 0, N.BFLOAT16, st) == N.ERR_ARG


@pytest.mark.parametrize("rows,cols,dt", [(4096, 2048, torch.bfloat16), (300, 777, torch.bfloat16),
                                          (64, 1024, torch.float32), (5, 24, torch.float32)])
def test_add_rmsnorm_equals_add_then_norm(rows, cols, dt):
    """The fused residual add + RMSNorm returns exactly what the add (rounded to the dtype)
    followed by nkl_rmsnorm returns, for the vectorised and the two-pass shapes."""
    from nkilab import ops

    g = torch.Generator().manual_seed(rows + cols)
    x = torch.randn(rows, cols, generator=g).to(dt).cuda()
    r = torch.randn(rows, cols, generator=g).to(dt).cuda()
    w = (1 + 0.1 * torch.randn(cols, generator=g)).to(dt).cuda()
    s, y = torch.ops.nkilab.add_rmsnorm(x, r, w, 1e-6)
    s_ref = x + r
    assert torch.equal(s, s_ref)
    assert torch.equal(y, ops.rmsnorm(s_ref, w, 1e-6))

"""Pin the CPU oracle (oracle/nki_oracle.py) before trusting it (CPU only).

1. Against every golden vector in tests/golden/ -- outputs of the reference's own
   kernel and host-wrapper source (see tests/golden/make_golden.py).
2. Against the PyTorch references and tolerances of the reference's tests
   (tests/test_attention.py, test_matmul.py, test_norm.py, test_model.py).
3. Against the reference tests' known-answer checks.
"""
from __future__ import annotations

import json
import math
import os

import ml_dtypes
import numpy as np
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from conftest import GOLDEN, bf16_ulp_diff, cases, load_golden, rel_err, to_numpy, to_torch
from oracle import nki_oracle as O

BF16 = ml_dtypes.bfloat16
ATT = load_golden("golden_attention.npz")
MM = load_golden("golden_matmul.npz")
NORM = load_golden("golden_norm.npz")
MODEL = load_golden("golden_model.npz")


def assert_matches_golden(out: np.ndarray, gold: np.ndarray, fp32_rel=1e-5, bf16_max_ulp=1, bf16_frac=0.01):
    assert out.shape == gold.shape and out.dtype == gold.dtype
    if gold.dtype == BF16:
        d = bf16_ulp_diff(out, gold)
        assert d.max() <= bf16_max_ulp, f"max ulp diff {d.max()}"
        assert (d > 0).mean() <= bf16_frac, f"{(d > 0).mean():.4f} of elements differ"
    else:
        assert rel_err(out, gold) < fp32_rel


# ------------------------------------------------------------------ golden vectors

@pytest.mark.parametrize("case", cases(ATT))
def test_attention_oracle_matches_reference_kernels(case):
    q, k, v = (to_torch(ATT[f"{case}/{n}"]) for n in "qkv")
    outs = [key for key in ATT if key.startswith(case + "/out_")]
    assert outs
    for key in outs:
        variant = key.split("/out_")[1]
        fn = O.attention_naive if variant == "naive" else O.attention_flash
        got = to_numpy(fn(q, k, v))
        # bf16: P is rounded inside the kernel, so one input-rounding flip can move an
        # output by a few ulps; the reference's own variants differ the same way.
        assert_matches_golden(got, ATT[key], bf16_max_ulp=4, bf16_frac=0.02)


@pytest.mark.parametrize("case", cases(MM))
def test_matmul_oracle_matches_reference_kernels(case):
    a, b = to_torch(MM[f"{case}/a"]), to_torch(MM[f"{case}/b"])
    got = to_numpy(O.matmul(a, b))
    for var in ("blocked", "naive"):
        assert_matches_golden(got, MM[f"{case}/out_{var}"])


@pytest.mark.parametrize("case", [c for c in cases(NORM) if c.startswith("softmax")])
def test_softmax_oracle_matches_reference_kernels(case):
    x = to_torch(NORM[f"{case}/x"])
    assert_matches_golden(to_numpy(O.softmax_fused(x)), NORM[f"{case}/out_fused"])
    assert_matches_golden(to_numpy(O.softmax_unfused(x)), NORM[f"{case}/out_unfused"])


@pytest.mark.parametrize("case", [c for c in cases(NORM) if c.startswith("rmsnorm")])
def test_rmsnorm_oracle_matches_reference_kernels(case):
    x, w = to_torch(NORM[f"{case}/x"]), to_torch(NORM[f"{case}/w"])
    assert_matches_golden(to_numpy(O.rmsnorm(x, w)), NORM[f"{case}/out"])


@pytest.mark.parametrize("case", [c for c in cases(NORM) if c.startswith("swiglu")])
def test_swiglu_oracle_matches_reference_kernels(case):
    g, u = to_torch(NORM[f"{case}/gate"]), to_torch(NORM[f"{case}/up"])
    assert_matches_golden(to_numpy(O.swiglu(g, u)), NORM[f"{case}/out"])


def _block_weights():
    from nkilab.model import BlockConfig, DecoderBlock

    torch.manual_seed(0)
    return DecoderBlock(BlockConfig()).eval()


@pytest.mark.parametrize("case", cases(MODEL))
def test_decoder_block_oracle_matches_reference(case):
    block = _block_weights()
    sums = np.array([p.detach().double().sum().item() for p in block.parameters()])
    np.testing.assert_allclose(sums, MODEL[f"{case}/param_sums"], rtol=1e-12)  # same seeded weights
    x = to_torch(MODEL[f"{case}/x"])
    got = O.decoder_block(x, block.norm1.weight.detach(), block.wqkv.weight.detach(), block.wo.weight.detach(),
                          block.norm2.weight.detach(), block.wg.weight.detach(), block.wu.weight.detach(),
                          block.wd.weight.detach(), block.cfg.n_heads, block.cfg.eps,
                          naive_attention=case.endswith("naive"))
    gold = MODEL[f"{case}/out_nki_forward"]
    if gold.dtype == BF16:
        assert rel_err(to_numpy(got).astype(np.float32), gold.astype(np.float32)) < 2e-2
    else:
        assert rel_err(to_numpy(got), gold) < 1e-5
        np.testing.assert_allclose(to_numpy(got), MODEL[f"{case}/out_torch_block"], atol=1e-5)


def test_choose_blocks_matches_reference_table():
    with open(os.path.join(GOLDEN, "golden_blocks.json")) as f:
        table = json.load(f)
    for key, want in table.items():
        m, n = map(int, key.split(","))
        assert list(O.choose_blocks(m, n)) == want


# ------------------------------------------------------------------ reference tests' torch references

def _sdpa(q, k, v):
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)


@pytest.mark.parametrize("variant", ["naive", "flash"])
@pytest.mark.parametrize("H,S,d", [(1, 128, 64), (2, 512, 64), (2, 200, 32), (1, 384, 128)])
def test_oracle_attention_vs_sdpa_fp32(rng, variant, H, S, d):
    q, k, v = (torch.from_numpy(rng.standard_normal((H, S, d)).astype(np.float32)) for _ in range(3))
    fn = O.attention_naive if variant == "naive" else O.attention_flash
    np.testing.assert_allclose(fn(q, k, v).numpy(), _sdpa(q, k, v).numpy(), atol=2e-5)


@pytest.mark.parametrize("variant", ["naive", "flash"])
def test_oracle_attention_bf16(rng, variant):
    q, k, v = (to_torch(rng.standard_normal((2, 256, 64)).astype(BF16)) for _ in range(3))
    ref = _sdpa(q.float(), k.float(), v.float()).numpy()
    fn = O.attention_naive if variant == "naive" else O.attention_flash
    assert rel_err(fn(q, k, v).float().numpy(), ref) < 3e-2


def test_oracle_first_token_attends_only_to_itself(rng):
    q, k, v = (torch.from_numpy(rng.standard_normal((1, 256, 64)).astype(np.float32)) for _ in range(3))
    np.testing.assert_allclose(O.attention_flash(q, k, v)[0, 0].numpy(), v[0, 0].numpy(), atol=1e-6)


@pytest.mark.parametrize("M,K,N", [(128, 128, 512), (256, 384, 1024), (200, 300, 130), (1, 7, 3)])
def test_oracle_matmul_fp32(rng, M, K, N):
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((K, N)).astype(np.float32)
    assert rel_err(O.matmul(torch.from_numpy(a), torch.from_numpy(b)).numpy(), a @ b) < 1e-5


@pytest.mark.parametrize("R,D", [(128, 64), (1000, 2048), (5, 3)])
def test_oracle_softmax_vs_torch(rng, R, D):
    x = torch.from_numpy((rng.standard_normal((R, D)) * 4).astype(np.float32))
    for fn in (O.softmax_fused, O.softmax_unfused):
        np.testing.assert_allclose(fn(x).numpy(), torch.softmax(x, -1).numpy(), rtol=1e-5, atol=1e-6)


def test_oracle_softmax_large_logits(rng):
    x = torch.from_numpy((rng.standard_normal((256, 512)) * 1e4).astype(np.float32))
    out = O.softmax_fused(x).numpy()
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out.sum(-1), 1.0, atol=1e-5)


@settings(max_examples=10, deadline=None)
@given(R=st.integers(1, 400), D=st.integers(1, 1024), s=st.floats(0.1, 50))
def test_oracle_softmax_rows_sum_to_one(R, D, s):
    x = torch.from_numpy((np.random.default_rng(R * 7 + D).standard_normal((R, D)) * s).astype(np.float32))
    out = O.softmax_fused(x).numpy()
    np.testing.assert_allclose(out.sum(-1), 1.0, atol=1e-5)
    assert (out >= 0).all()


@pytest.mark.parametrize("R,D", [(128, 256), (300, 1024), (7, 33)])
def test_oracle_rmsnorm_vs_torch(rng, R, D):
    x = rng.standard_normal((R, D)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, D).astype(np.float32)
    xt = torch.from_numpy(x)
    ref = (xt * torch.rsqrt(xt.pow(2).mean(-1, keepdim=True) + 1e-6) * torch.from_numpy(w)).numpy()
    assert rel_err(O.rmsnorm(xt, torch.from_numpy(w)).numpy(), ref) < 1e-5


def test_oracle_swiglu_vs_torch(rng):
    g = torch.from_numpy(rng.standard_normal((300, 1024)).astype(np.float32))
    u = torch.from_numpy(rng.standard_normal((300, 1024)).astype(np.float32))
    ref = (torch.nn.functional.silu(g) * u).numpy()
    assert rel_err(O.swiglu(g, u).numpy(), ref) < 1e-5


def test_oracle_flash_equals_scaled_definition():
    """The flash restatement is exact attention: compare with a float64 softmax."""
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(2, 300, 64, generator=g) for _ in range(3))
    s = (q.double() @ k.double().transpose(1, 2)) / math.sqrt(64)
    s = s.masked_fill(torch.triu(torch.ones(300, 300, dtype=torch.bool), 1), float("-inf"))
    ref = torch.softmax(s, -1) @ v.double()
    np.testing.assert_allclose(O.attention_flash(q, k, v).numpy(), ref.numpy(), atol=2e-5)

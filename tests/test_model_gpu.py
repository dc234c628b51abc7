"""GPU parity of the decoder block (nkilab.model.nki_forward on the CUDA kernels)."""
from __future__ import annotations

import ml_dtypes
import numpy as np
import pytest
import torch

from conftest import bf16_excess_rel, cases, load_golden, rel_err, to_numpy, to_torch
from oracle import nki_oracle as O

pytestmark = pytest.mark.gpu
BF16 = ml_dtypes.bfloat16
MODEL = load_golden("golden_model.npz")


def _block(cfg=None, seed=0):
    from nkilab.model import BlockConfig, DecoderBlock

    torch.manual_seed(seed)
    return DecoderBlock(cfg or BlockConfig()).eval()


def _oracle(block, x):
    return O.decoder_block(x, block.norm1.weight.detach(), block.wqkv.weight.detach(), block.wo.weight.detach(),
                           block.norm2.weight.detach(), block.wg.weight.detach(), block.wu.weight.detach(),
                           block.wd.weight.detach(), block.cfg.n_heads, block.cfg.eps)


@pytest.mark.parametrize("case", cases(MODEL))
def test_decoder_block_matches_reference(case):
    from nkilab.model import nki_forward

    block = _block()
    x = MODEL[f"{case}/x"]
    variant = "naive" if case.endswith("naive") else "flash_pipelined"
    out = nki_forward(block, x, attention_variant=variant)
    gold = MODEL[f"{case}/out_nki_forward"]
    if gold.dtype == BF16:
        assert out.dtype == BF16
        # north_star's 3e-3, net of the final bf16 rounding of the output (see bf16_excess_rel)
        assert bf16_excess_rel(out, gold) < 3e-3
        assert rel_err(out.astype(np.float32), gold.astype(np.float32)) < 1e-2
    else:
        np.testing.assert_allclose(out, MODEL[f"{case}/out_torch_block"], atol=1e-5)
        assert rel_err(out, gold) < 1e-5


@pytest.mark.parametrize("S", [128, 300])
@pytest.mark.parametrize("variant", ["naive", "flash_pipelined"])
def test_decoder_block_matches_pytorch(S, variant):
    """tests/test_model.py:8-17 of the reference."""
    from nkilab.model import nki_forward

    block = _block()
    x = torch.randn(S, block.cfg.d_model)
    with torch.no_grad():
        ref = block(x).numpy()
    np.testing.assert_allclose(nki_forward(block, x.numpy(), attention_variant=variant), ref, atol=1e-5)


def _oracle_pair(block, x):
    """The oracle block with fp32 accumulation (the reference's arithmetic) and with
    fp64 accumulation (same bf16 rounding points, no accumulation error)."""
    ws = [getattr(block, n).weight.detach() for n in ("norm1", "wqkv", "wo", "norm2", "wg", "wu", "wd")]
    o32 = O.decoder_block(x, *ws, block.cfg.n_heads, block.cfg.eps)
    o64 = O.decoder_block(x, *ws, block.cfg.n_heads, block.cfg.eps, acc=torch.float64)
    return o32.float().numpy(), o64.float().numpy()


def assert_block_parity(got, o32, o64, bar=3e-3):
    """north_star's bar for the bf16 block: rel_err(gpu, oracle) <= 3e-3. A bf16 block
    rounds its activations at every stage, so two correct fp32-accumulating
    implementations differ by output ulps; where that floor -- measured here on the same
    inputs as the distance between the fp32 oracle and the fp64-accumulated oracle --
    exceeds 3e-3, the GPU must stay within 1.25x of it, measured against either oracle."""
    err32, err64 = rel_err(got, o32), rel_err(got, o64)
    floor = rel_err(o32, o64)
    # element statistics beside the max: mean |error| and the share of elements that
    # differ from the fp64-accumulated oracle, for the GPU and for the fp32 oracle
    g64, f64 = np.abs(got - o64), np.abs(o32 - o64)
    msg = (f"gpu vs fp32 oracle {err32:.3e}, gpu vs fp64 oracle {err64:.3e}, "
           f"floor (fp32 vs fp64 oracle) {floor:.3e}; mean |err| vs fp64: gpu {g64.mean():.3e}, "
           f"fp32 oracle {f64.mean():.3e}; elements differing: gpu {(g64 > 0).mean():.2e}, "
           f"fp32 oracle {(f64 > 0).mean():.2e}")
    print(msg)
    if floor <= bar:
        assert err32 <= bar, msg
    else:
        assert min(err32, err64) <= 1.25 * floor, msg
    return err32, err64, floor


def test_decoder_block_device_batched_bf16():
    """Device path with a batch dimension vs per-sequence oracle results at north_star's
    3e-3 (or 1.25x the measured fp32-vs-fp64 floor). d_ff is a multiple of 128, so the
    block runs the fused gate/up + SwiGLU GEMM."""
    from nkilab.model import BlockConfig, nki_forward

    block = _block(BlockConfig(d_model=512, n_heads=4, d_ff=1408))
    g = torch.Generator().manual_seed(4)
    x = torch.randn(2, 384, 512, generator=g).to(torch.bfloat16)
    out = nki_forward(block, x.cuda())
    assert "wgu" in block.__dict__["_nkl_weight_cache"][(torch.bfloat16, "cuda:0")][1]
    assert out.shape == x.shape and out.dtype == torch.bfloat16
    for b in range(2):
        o32, o64 = _oracle_pair(block, x[b])
        assert_block_parity(out[b].float().cpu().numpy(), o32, o64)


def test_decoder_block_baseline_config_bf16():
    """BASELINE configs[4], the block bench.py times: B=4, S=4096, d=4096, 32 heads x 128,
    d_ff=11008 (a multiple of 128: fused gate/up + SwiGLU GEMM), bf16 weights ~ N(0, 0.02),
    norm gains ~ U(0.5, 1.5), x ~ N(0, 1). The device path runs the whole batch (strided
    attention over the fused QKV projection, add + RMSNorm, residual in the down-projection
    epilogue); the first and last batch elements are compared with the CPU oracle
    (nkilab/model.py:70-89) at north_star's bar."""
    from nkilab.model import BlockConfig, DecoderBlock, nki_forward

    cfg = BlockConfig(d_model=4096, n_heads=32, d_ff=11008)
    with torch.device("meta"):
        block = DecoderBlock(cfg)
    block = block.to_empty(device="cpu").eval()
    g = torch.Generator().manual_seed(2024)
    with torch.no_grad():
        for n in ("wqkv", "wo", "wg", "wu", "wd"):
            getattr(block, n).weight.normal_(0.0, 0.02, generator=g)
        for n in ("norm1", "norm2"):
            getattr(block, n).weight.uniform_(0.5, 1.5, generator=g)
    x = torch.randn(4, 4096, 4096, generator=g).to(torch.bfloat16)
    out = nki_forward(block, x.cuda()).cpu()
    block.__dict__.pop("_nkl_weight_cache", None)  # release the device weights
    torch.cuda.empty_cache()
    assert out.shape == x.shape and out.dtype == torch.bfloat16
    for b in (0, 3):
        o32, o64 = _oracle_pair(block, x[b])
        assert_block_parity(out[b].float().numpy(), o32, o64)


def test_decoder_block_stages_teacher_forced_bf16():
    """north_star's bf16 bar (3e-3) stage by stage: every kernel of the block, fed the
    oracle's own input for that stage, matches the oracle's output for it (net of one
    ulp for the stage's output rounding)."""
    from nkilab import ops

    block = _block(BlockConfig_small())
    bf = torch.bfloat16
    x = torch.randn(384, 512, generator=torch.Generator().manual_seed(5)).to(bf)
    W = {n: getattr(block, n).weight.detach().t().contiguous().to(bf) for n in ("wqkv", "wo", "wg", "wu", "wd")}
    g1, g2 = block.norm1.weight.detach().to(bf), block.norm2.weight.detach().to(bf)
    c = lambda t: t.cuda()  # noqa: E731

    def check(gpu, ref):
        a, b = gpu.float().cpu().numpy(), ref.float().numpy()
        assert bf16_excess_rel(a, b) < 3e-3, bf16_excess_rel(a, b)

    h = O.rmsnorm(x, g1)
    check(ops.rmsnorm(c(x), c(g1)), h)
    qkv = O.matmul(h, W["wqkv"])
    check(ops.matmul(c(h), c(W["wqkv"])), qkv)
    q, k, v = (qkv[:, i * 512:(i + 1) * 512].reshape(384, 4, 128).transpose(0, 1).contiguous() for i in range(3))
    a = O.attention_flash(q, k, v)
    check(ops.attention(c(q), c(k), c(v)), a)
    am = a.transpose(0, 1).reshape(384, 512).contiguous()
    wo = O.matmul(am, W["wo"])
    check(ops.matmul(c(am), c(W["wo"])), wo)
    x1 = (x.float() + wo.float()).to(bf)
    h2 = O.rmsnorm(x1, g2)
    check(ops.rmsnorm(c(x1), c(g2)), h2)
    gg, uu = O.matmul(h2, W["wg"]), O.matmul(h2, W["wu"])
    check(ops.matmul(c(h2), c(W["wg"])), gg)
    check(ops.matmul(c(h2), c(W["wu"])), uu)
    act = O.swiglu(gg, uu)
    check(ops.swiglu(c(gg), c(uu)), act)
    check(ops.matmul(c(act), c(W["wd"])), O.matmul(act, W["wd"]))


def BlockConfig_small():
    from nkilab.model import BlockConfig

    return BlockConfig(d_model=512, n_heads=4, d_ff=1376)


def test_weight_cache_refreshes_on_update():
    from nkilab.model import nki_forward

    block = _block()
    x = torch.randn(128, 256).cuda()
    y1 = nki_forward(block, x)
    with torch.no_grad():
        block.wd.weight.mul_(0.0)
    y2 = nki_forward(block, x)
    assert not torch.equal(y1, y2)

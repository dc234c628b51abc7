"""GPU parity of causal attention (tcgen05 flash bf16, exact fp32 flash, naive)."""
from __future__ import annotations

import math

import ml_dtypes
import numpy as np
import pytest
import torch

from conftest import bf16_ulp_diff, cases, load_golden, rel_err, to_numpy, to_torch
from oracle import nki_oracle as O

pytestmark = pytest.mark.gpu
BF16 = ml_dtypes.bfloat16
ATT = load_golden("golden_attention.npz")
FLASH = ["flash", "flash_kv_resident", "flash_balanced", "flash_pipelined"]


@pytest.fixture(scope="module")
def ops():
    from nkilab import ops as _ops

    return _ops


def _sdpa(q, k, v):
    return torch.nn.functional.scaled_dot_product_attention(*map(torch.from_numpy, (q, k, v)), is_causal=True).numpy()


@pytest.mark.parametrize("case", cases(ATT))
def test_attention_matches_reference_golden(ops, case):
    q, k, v = (ATT[f"{case}/{n}"] for n in "qkv")
    for key in [k_ for k_ in ATT if k_.startswith(case + "/out_")]:
        variant = key.split("/out_")[1]
        out = ops.attention(q, k, v, variant=variant)
        gold = ATT[key]
        assert out.shape == gold.shape and out.dtype == gold.dtype
        if gold.dtype == BF16:
            assert rel_err(out.astype(np.float32), gold.astype(np.float32)) < 3e-3, variant
        else:
            np.testing.assert_allclose(out, gold, atol=2e-5)


@pytest.mark.parametrize("variant", ["naive"] + FLASH)
@pytest.mark.parametrize("H,S,d", [(1, 128, 64), (2, 512, 64), (2, 200, 32), (1, 384, 128)])
def test_attention_matches_torch_fp32(ops, rng, variant, H, S, d):
    q, k, v = (rng.standard_normal((H, S, d)).astype(np.float32) for _ in range(3))
    out = ops.attention(q, k, v, variant=variant)
    assert out.shape == (H, S, d)
    np.testing.assert_allclose(out, _sdpa(q, k, v), atol=2e-5)


@pytest.mark.parametrize("variant", ["naive", "flash_pipelined"])
def test_attention_bf16(ops, rng, variant):
    q, k, v = (rng.standard_normal((2, 256, 64)).astype(BF16) for _ in range(3))
    ref = _sdpa(*(t.astype(np.float32) for t in (q, k, v)))
    assert rel_err(ops.attention(q, k, v, variant=variant).astype(np.float32), ref) < 3e-2


def test_first_token_attends_only_to_itself(ops, rng):
    q, k, v = (rng.standard_normal((1, 256, 64)).astype(np.float32) for _ in range(3))
    out = ops.attention(q, k, v)
    np.testing.assert_allclose(out[0, 0], v[0, 0], atol=1e-6)


@pytest.mark.parametrize("dtype", [np.float32, BF16])
def test_variants_agree_bitwise_on_flash_family(ops, rng, dtype):
    q, k, v = (rng.standard_normal((2, 512, 64)).astype(dtype) for _ in range(3))
    outs = [ops.attention(q, k, v, variant=n) for n in ("flash_balanced", "flash_pipelined")]
    np.testing.assert_array_equal(outs[0].view(np.uint8), outs[1].view(np.uint8))


def _check_vs_oracle(out_dev, q, k, v, rel=3e-3):
    ref = O.attention_flash(q, k, v)
    got = out_dev.float().cpu().numpy()
    assert rel_err(got, ref.float().numpy()) < rel


@pytest.mark.parametrize("H,S", [(8, 2048), (1, 4096)])
def test_attention_baseline_configs(ops, H, S):
    """causal 8 x 2048 x 128 and 1 x 4096 x 128 bf16 vs the oracle."""
    g = torch.Generator().manual_seed(H * 10000 + S)
    q, k, v = (torch.randn(H, S, 128, generator=g).to(torch.bfloat16) for _ in range(3))
    out = ops.attention(q.cuda(), k.cuda(), v.cuda())
    _check_vs_oracle(out, q, k, v)


@pytest.mark.parametrize("H,S,d", [(1, 1, 128), (3, 129, 64), (2, 200, 128), (1, 257, 64), (2, 130, 32),
                                   (1, 640, 96), (4, 1000, 128)])
def test_attention_bf16_edge_shapes(ops, H, S, d):
    g = torch.Generator().manual_seed(H * 7 + S * 3 + d)
    q, k, v = (torch.randn(H, S, d, generator=g).to(torch.bfloat16) for _ in range(3))
    out = ops.attention(q.cuda(), k.cuda(), v.cuda())
    assert out.shape == (H, S, d)
    _check_vs_oracle(out, q, k, v)


def test_attention_is_causal(ops):
    """Changing keys/values after position t leaves outputs up to t unchanged (bitwise)."""
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn(2, 1024, 128, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    out1 = ops.attention(q, k, v)
    k2, v2 = k.clone(), v.clone()
    k2[:, 600:] = torch.randn_like(k2[:, 600:].float()).to(torch.bfloat16)
    v2[:, 600:] = 7.0
    out2 = ops.attention(q, k2, v2)
    assert torch.equal(out1[:, :600], out2[:, :600])
    assert not torch.equal(out1[:, 600:], out2[:, 600:])


def test_attention_rows_are_convex_combinations(ops):
    """With v = const c in one column, that output column equals c (softmax rows sum to 1)."""
    g = torch.Generator().manual_seed(12)
    q, k = (torch.randn(4, 2048, 128, generator=g).to(torch.bfloat16).cuda() for _ in range(2))
    v = torch.randn(4, 2048, 128, generator=g).to(torch.bfloat16).cuda()
    v[..., 5] = 0.5
    out = ops.attention(q, k, v)
    np.testing.assert_allclose(out[..., 5].float().cpu().numpy(), 0.5, atol=4e-3)


def test_kernel_level_layout(rng):
    """The reference's kernel-level layout: qT, kT [H, d, S], v [H, S, d]."""
    from nkilab.kernels import attention as at

    q, k, v = (rng.standard_normal((2, 256, 64)).astype(np.float32) for _ in range(3))
    qT, kT = (np.ascontiguousarray(t.transpose(0, 2, 1)) for t in (q, k))
    for fn in (at.attention_naive, at.flash_attention, at.flash_attention_pipelined):
        np.testing.assert_allclose(fn(qT, kT, v, 1 / 8.0), _sdpa(q, k, v), atol=2e-5)


def test_device_flag_clean_after_runs():
    from nkilab import _native as N

    N.check_device(torch.cuda.current_stream().cuda_stream)


def test_split_kv_workspace_path_matches_single_unit_path():
    """nkl_attention_ws (key range split over SMs, partials combined by a second kernel)
    vs nkl_attention (one unit per query tile) through the C ABI, repeatable call to call,
    and independent of what the workspace held before (it needs no zeroing)."""
    import ctypes
    import math

    from nkilab import _native as N

    g = torch.Generator().manual_seed(21)
    H, S, D = 8, 2048, 128
    q, k, v = (torch.randn(H, S, D, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    nbytes = N.lib.nkl_attention_workspace_size(H, S, D, N.BFLOAT16)
    assert nbytes > 0  # 128 query tiles do not fill 148 SMs: the split path is taken
    ws = torch.full((nbytes,), 0xA5, dtype=torch.uint8, device="cuda")
    o1, o2, o3 = (torch.empty_like(q) for _ in range(3))
    scale = 1 / math.sqrt(D)
    assert N.lib.nkl_attention(p(q), p(k), p(v), p(o1), H, S, D, scale, N.BFLOAT16, st) == N.OK
    for o in (o2, o3):
        assert N.lib.nkl_attention_ws(p(q), p(k), p(v), p(o), p(ws), nbytes, H, S, D, scale, N.BFLOAT16, st) == N.OK
    N.check_device(st.value)
    assert torch.equal(o2, o3)  # combine order is fixed: bit-identical across calls
    assert rel_err(o2.float().cpu().numpy(), o1.float().cpu().numpy()) < 3e-3
    _check_vs_oracle(o2, q.cpu(), k.cpu(), v.cpu())


@pytest.mark.parametrize("H,Hkv,S,D,dt", [(8, 2, 2048, 128, torch.bfloat16), (8, 1, 1000, 64, torch.bfloat16),
                                          (4, 2, 300, 96, torch.bfloat16), (4, 1, 257, 64, torch.float32)])
def test_grouped_query_attention_equals_repeated_heads(H, Hkv, S, D, dt):
    """k, v with Hkv heads: query head h uses key/value head h // (H // Hkv). The result
    equals plain attention on k, v with each head repeated H // Hkv times (same kernel,
    same data), bit for bit, and the oracle within the attention tolerance."""
    from nkilab import ops

    g = torch.Generator().manual_seed(H * 1000 + Hkv * 100 + S)
    q = torch.randn(H, S, D, generator=g).to(dt)
    k = torch.randn(Hkv, S, D, generator=g).to(dt)
    v = torch.randn(Hkv, S, D, generator=g).to(dt)
    rep = H // Hkv
    got = ops.attention(q.cuda(), k.cuda(), v.cuda())
    full = ops.attention(q.cuda(), k.repeat_interleave(rep, 0).cuda(), v.repeat_interleave(rep, 0).cuda())
    assert torch.equal(got, full)
    if dt == torch.float32:
        ref = torch.nn.functional.scaled_dot_product_attention(q, k.repeat_interleave(rep, 0), v.repeat_interleave(rep, 0),
                                                               is_causal=True)
        assert float((got.cpu() - ref).abs().max()) < 2e-5
    else:
        ref = O.attention_flash(q[:2], k.repeat_interleave(rep, 0)[:2], v.repeat_interleave(rep, 0)[:2])
        assert rel_err(to_numpy(got[:2].cpu()), to_numpy(ref)) < 3e-3


def test_grouped_query_attention_rejects_bad_head_counts():
    from nkilab import _native as N

    q = torch.zeros(6, 128, 64, dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros(4, 128, 64, dtype=torch.bfloat16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = N.lib.nkl_attention_gqa(q.data_ptr(), kv.data_ptr(), kv.data_ptr(), q.data_ptr(), None, 0, 6, 4, 128, 64,
                                 0.125, N.BFLOAT16, st)
    assert rc == N.ERR_SHAPE and "kv_heads must divide heads" in N.lib.nkl_last_error().decode()


def test_split_kv_workspace_under_cuda_graph_replay():
    """The split path (attention kernel + combine kernel) captured once in a CUDA graph
    and replayed on new inputs in the captured buffers: every replay matches an eager
    nkl_attention_ws call on the same inputs bit for bit, and the oracle."""
    import ctypes
    import math

    from nkilab import _native as N

    H, S, D = 8, 2048, 128
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.empty(H, S, D, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    nbytes = N.lib.nkl_attention_workspace_size(H, S, D, N.BFLOAT16)
    assert nbytes > 0
    ws_graph = torch.full((nbytes,), 0x5A, dtype=torch.uint8, device="cuda")
    ws_eager = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    o_graph, o_eager = torch.empty_like(q), torch.empty_like(q)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    scale = 1 / math.sqrt(D)

    def call(o, ws):
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        return N.lib.nkl_attention_ws(p(q), p(k), p(v), p(o), p(ws), nbytes, H, S, D, scale, N.BFLOAT16, st)

    for t in (q, k, v):
        t.copy_(torch.randn(H, S, D, generator=g).to(torch.bfloat16))
    assert call(o_graph, ws_graph) == N.OK  # plan and kernel attributes set up before capture
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        assert call(o_graph, ws_graph) == N.OK
    for trial in range(3):
        for t in (q, k, v):
            t.copy_(torch.randn(H, S, D, generator=g).to(torch.bfloat16))
        o_graph.fill_(float("nan"))
        graph.replay()
        assert call(o_eager, ws_eager) == N.OK
        torch.cuda.synchronize()
        N.check_device(torch.cuda.current_stream().cuda_stream)
        assert torch.equal(o_graph, o_eager), f"replay {trial}"
    _check_vs_oracle(o_graph, q.cpu(), k.cpu(), v.cpu())



def test_graphs_captured_with_default_settings_replay_concurrently():
    """Two CUDA graphs of the split-KV attention op, captured with torch.cuda.graph's
    defaults (one shared capture stream), replayed at the same time on two streams: each
    graph owns the workspace it captured, so the replays do not race and each matches an
    eager call on its own inputs bit for bit."""
    H, S, D = 8, 2048, 128
    g = torch.Generator(device="cuda").manual_seed(17)
    ins = [[torch.randn(H, S, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3)] for _ in range(2)]
    scale = 1.0 / math.sqrt(D)
    for t in ins:  # plan and kernel attributes set up before capture
        torch.ops.nkilab.attention(*t, scale, False)
    torch.cuda.synchronize()
    graphs, outs = [], []
    for t in ins:
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            outs.append(torch.ops.nkilab.attention(*t, scale, False))
        graphs.append(gr)
    ref = [torch.ops.nkilab.attention(*t, scale, False) for t in ins]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for _ in range(5):
        for o in outs:
            o.fill_(float("nan"))
        torch.cuda.synchronize()
        for gr, st in zip(graphs, streams):
            with torch.cuda.stream(st):
                for _ in range(4):
                    gr.replay()
        torch.cuda.synchronize()
        for o, r in zip(outs, ref):
            assert torch.equal(o, r)


@pytest.mark.parametrize("H,Hkv,S,D", [(8, 8, 2048, 128), (32, 32, 1000, 128), (8, 2, 700, 64)])
def test_strided_attention_matches_contiguous_bit_for_bit(ops, H, Hkv, S, D):
    """nkl_attention_strided reading q/k/v straight out of a fused [S, q|k|v, heads, d]
    projection and writing out as [S, H, d]: the same kernels on the same plan as the
    contiguous entry point, so the same bits (split-KV combine included at 8x2048)."""
    g = torch.Generator(device="cuda").manual_seed(H + S)
    width = (H + 2 * Hkv) * D
    qkv = torch.randn(S, width, device="cuda", generator=g).to(torch.bfloat16)
    q = qkv[:, :H * D].view(S, H, D).transpose(0, 1)
    k = qkv[:, H * D:(H + Hkv) * D].view(S, Hkv, D).transpose(0, 1)
    v = qkv[:, (H + Hkv) * D:].view(S, Hkv, D).transpose(0, 1)
    o = torch.full((S, H, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    torch.ops.nkilab.attention_strided_(q, k, v, o.transpose(0, 1), 1.0 / math.sqrt(D))
    ref = ops.attention(q.contiguous(), k.contiguous(), v.contiguous())
    torch.cuda.synchronize()
    assert torch.equal(o.transpose(0, 1), ref)

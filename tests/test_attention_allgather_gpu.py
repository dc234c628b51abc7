"""nkl_attention_allgather on one GPU: with one rank it is plain attention into the full
output buffer; with a second rank that never takes part, the flag exchange's bounded wait
runs out, the kernel returns, nkl_check_device reports NKL_ERR_DEVICE and the context stays
usable. (The two-rank exchange itself runs in tests/test_parallel_nccl.py on two GPUs.)"""
from __future__ import annotations

import ctypes
import math
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

H, S, D = 8, 2048, 128


@pytest.fixture(autouse=True)
def _torch_ops():
    from nkilab import ops  # noqa: F401  (registers torch.ops.nkilab)


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _call(N, q, k, v, outs, flags, world, rank, heads_total, head_offset):
    heads = q.shape[0]
    nbytes = N.lib.nkl_attention_workspace_size(heads, S, D, N.BFLOAT16)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
    arr = ctypes.c_void_p * world
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return N.lib.nkl_attention_allgather(_p(q), _p(k), _p(v), arr(*[o.data_ptr() for o in outs]),
                                         arr(*[f.data_ptr() for f in flags]), world, rank, heads_total, head_offset,
                                         _p(ws), nbytes, heads, S, D, 1.0 / math.sqrt(D), N.BFLOAT16, st)


def test_single_rank_is_plain_attention():
    from nkilab import _native as N

    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = (torch.randn(H, S, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    out = torch.full((H, S, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    flags = torch.zeros(64, dtype=torch.int32, device="cuda")
    assert _call(N, q, k, v, [out], [flags], 1, 0, H, 0) == N.OK, N.lib.nkl_last_error()
    ref = torch.ops.nkilab.attention(q, k, v, 1.0 / math.sqrt(D), False)
    torch.cuda.synchronize()
    N.check_device(torch.cuda.current_stream().cuda_stream)
    assert torch.equal(out, ref)


def test_heads_land_at_their_offset():
    """Three of eight heads written at head offset 5 of an 8-head buffer; the other heads
    are untouched."""
    from nkilab import _native as N

    g = torch.Generator(device="cuda").manual_seed(4)
    q, k, v = (torch.randn(3, S, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    out = torch.zeros((H, S, D), dtype=torch.bfloat16, device="cuda")
    flags = torch.zeros(64, dtype=torch.int32, device="cuda")
    assert _call(N, q, k, v, [out], [flags], 1, 0, H, 5) == N.OK, N.lib.nkl_last_error()
    ref = torch.ops.nkilab.attention(q, k, v, 1.0 / math.sqrt(D), False)
    torch.cuda.synchronize()
    assert torch.equal(out[5:], ref)
    assert torch.count_nonzero(out[:5]) == 0


def test_missing_peer_times_out_and_reports():
    """world = 2 with rank 1 absent: rank 1's 'buffers' are ordinary allocations on this GPU
    that nothing signals, so the exchange's wait for rank 1's count expires after its ~1 s
    limit. The call's kernels all return; the failure comes back as NKL_ERR_DEVICE."""
    from nkilab import _native as N

    g = torch.Generator(device="cuda").manual_seed(5)
    q, k, v = (torch.randn(4, S, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    outs = [torch.zeros((H, S, D), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    flags = [torch.zeros(64, dtype=torch.int32, device="cuda") for _ in range(2)]
    st = torch.cuda.current_stream().cuda_stream
    t0 = time.time()
    assert _call(N, q, k, v, outs, flags, 2, 0, H, 0) == N.OK, N.lib.nkl_last_error()
    rc = N.lib.nkl_check_device(ctypes.c_void_p(st))
    waited = time.time() - t0
    assert rc == N.ERR_DEVICE, rc
    assert b"attention code 90" in N.lib.nkl_last_error()
    assert 0.5 < waited < 30.0, waited
    # this rank announced itself in rank 1's array and counted the call; its heads reached
    # both buffers before the exchange
    assert int(flags[1][0]) == 1 and int(flags[0][2]) == 1
    ref = torch.ops.nkilab.attention(q, k, v, 1.0 / math.sqrt(D), False)
    torch.cuda.synchronize()
    assert torch.equal(outs[0][:4], ref) and torch.equal(outs[1][:4], ref)
    # the context is still usable and the device flag was cleared by the check
    assert N.lib.nkl_check_device(ctypes.c_void_p(st)) == N.OK
    assert torch.equal(torch.ops.nkilab.attention(q, k, v, 1.0 / math.sqrt(D), False), ref)


def test_argument_checks():
    from nkilab import _native as N

    t = torch.zeros(8, dtype=torch.int32, device="cuda")
    arr = (ctypes.c_void_p * 1)(t.data_ptr())
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = (_p(t), _p(t), _p(t), arr, arr)
    assert N.lib.nkl_attention_allgather(*args, 9, 0, 8, 0, None, 0, 8, S, D, 0.1, N.BFLOAT16, st) == N.ERR_ARG
    assert N.lib.nkl_attention_allgather(*args, 1, 1, 8, 0, None, 0, 8, S, D, 0.1, N.BFLOAT16, st) == N.ERR_ARG
    assert N.lib.nkl_attention_allgather(*args, 1, 0, 8, 6, None, 0, 4, S, D, 0.1, N.BFLOAT16, st) == N.ERR_SHAPE
    assert N.lib.nkl_attention_allgather(*args, 1, 0, 8, 0, None, 0, 8, S, D, 0.1, N.FLOAT32, st) == N.ERR_DTYPE

"""The allocation-free softmax entry point, nkl_softmax_unfused_static, through the C ABI.

Some callers of this library cannot call cudaMalloc: a host that binds only the C ABI
from a language runtime with no CUDA allocator binding, or one that must stay inside
a device-memory budget owned by another allocator. For them the unfused softmax has
a variant whose scratch is a fixed array inside the library's device image instead
of a caller-supplied workspace. These tests check that it gives the same result as
the workspace entry point, nkl_softmax_unfused, on two calls in a row (the second call
reuses scratch the first one left behind), and that it refuses inputs whose scratch
would not fit instead of launching.

This file is named so that pytest collects it last; it also passes when run alone in
a fresh process (the first call on a device does the one-time address lookup).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import nki_oracle as O

pytestmark = pytest.mark.gpu


def _p(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _codes():
    from nkilab import _native as N

    return N, {torch.float32: N.FLOAT32, torch.bfloat16: N.BFLOAT16}


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,cols", [(1000, 2048), (37, 333), (1, 8)])
def test_static_scratch_matches_workspace_entry_point(dtype, rows, cols):
    N, code = _codes()
    stream = torch.cuda.current_stream().cuda_stream
    st = ctypes.c_void_p(stream)
    nbytes = N.lib.nkl_softmax_unfused_workspace_size(rows, cols)
    assert nbytes <= N.SOFTMAX_UNFUSED_STATIC_BYTES
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    for call in range(2):  # two calls in a row: the second reuses the first call's scratch
        g = torch.Generator().manual_seed(100 * call + rows + cols)
        x = (torch.randn(rows, cols, generator=g) * (4.0 if call else 1.0)).to(dtype).cuda()
        y_static = torch.full_like(x, float("nan"))
        y_ws = torch.full_like(x, float("nan"))
        rc = N.lib.nkl_softmax_unfused_static(_p(x), _p(y_static), rows, cols, code[dtype], st)
        assert rc == N.OK, N.lib.nkl_last_error()
        rc = N.lib.nkl_softmax_unfused(_p(x), _p(y_ws), _p(ws), nbytes, rows, cols, code[dtype], st)
        assert rc == N.OK, N.lib.nkl_last_error()
        torch.cuda.synchronize()
        # the same three kernels on the same input: the same bits, and the oracle's
        # restatement of the reference's unfused softmax within the usual tolerance
        assert torch.equal(y_static, y_ws)
        a = y_static.float().cpu().numpy()
        assert np.isfinite(a).all()
        ref = O.softmax_unfused(x.cpu()).float().numpy()
        assert rel_err(a, ref) < (1e-5 if dtype == torch.float32 else 1e-2)
    N.check_device(stream)


def test_static_scratch_rejects_inputs_that_do_not_fit():
    N, code = _codes()
    rows, cols = 4096, 2048  # fp32 exponentials alone need 32 MiB
    assert N.lib.nkl_softmax_unfused_workspace_size(rows, cols) > N.SOFTMAX_UNFUSED_STATIC_BYTES
    x = torch.zeros(rows, cols, device="cuda")
    y = torch.zeros_like(x)
    rc = N.lib.nkl_softmax_unfused_static(_p(x), _p(y), rows, cols, code[torch.float32],
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == N.ERR_SHAPE
    assert b"scratch" in N.lib.nkl_last_error()
    torch.cuda.synchronize()
    assert torch.count_nonzero(y) == 0  # nothing was launched


@pytest.mark.parametrize("rows,cols", [(1, 1 << 62), (3, 1 << 61), (1 << 30, 1 << 33)])
def test_static_scratch_rejects_sizes_whose_byte_count_overflows(rows, cols):
    """rows * cols * 4 wraps around 64 bits for these shapes; the size check is done
    before any product is formed, so they are refused rather than launched. The
    pointers are never touched: the call returns before any launch."""
    N, code = _codes()
    y = torch.zeros(16, device="cuda")
    rc = N.lib.nkl_softmax_unfused_static(_p(y), _p(y), rows, cols, code[torch.float32],
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == N.ERR_SHAPE
    assert b"scratch" in N.lib.nkl_last_error()
    assert N.lib.nkl_softmax_unfused_workspace_size(rows, cols) == ctypes.c_size_t(-1).value
    torch.cuda.synchronize()
    assert torch.count_nonzero(y) == 0

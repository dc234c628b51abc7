"""GEMM in the reference's kernel-level form (nkilab/kernels/matmul.py).

The reference kernels take the left operand transposed (lhsT [K, M]) and the right
operand as rhs [K, N] and return out [M, N] in lhsT's dtype, with shapes already
padded to the tile multiples TK, TM, TN. These functions keep that contract and the
reference's asserts; the product itself runs on the B200 GEMM kernels, which read A
row-major, so lhsT is transposed on the device first.
"""
from __future__ import annotations

import torch

from .. import _torch_ops  # noqa: F401
from .._host import like_input, to_device

TK = 128  # contraction tile
TM = 128  # output rows per tile
TN = 512  # output columns per tile (one fp32 PSUM bank on Trainium2)


def _operands(lhsT, rhs):
    K, M = lhsT.shape
    K2, N = rhs.shape
    assert K == K2, (lhsT.shape, rhs.shape)
    a = to_device(lhsT).t().contiguous()
    b = to_device(rhs, a.device)
    if b.dtype != a.dtype:
        b = b.to(a.dtype)
    return a, b, K, M, N


def matmul_naive(lhsT, rhs):
    """Both operands re-read from memory for every (m, n, k) step (matmul.py:24-43)."""
    K, M = lhsT.shape
    N = rhs.shape[1]
    assert K % TK == 0 and M % TM == 0 and N % TN == 0
    a, b, *_ = _operands(lhsT, rhs)
    return like_input(torch.ops.nkilab.matmul(a, b, True), lhsT)


def matmul_blocked(lhsT, rhs, BM: int = 2, BN: int = 4):
    """Blocked GEMM (matmul.py:46-82); BM x BN output tiles of [TM, TN] must fit the
    8-bank PSUM budget of the reference, asserted with the reference's message."""
    K, M = lhsT.shape
    N = rhs.shape[1]
    assert K % TK == 0 and M % (TM * BM) == 0 and N % (TN * BN) == 0
    assert BM * BN <= 8, "BM*BN fp32 [128,512] accumulators must fit 8 PSUM banks"
    a, b, *_ = _operands(lhsT, rhs)
    return like_input(torch.ops.nkilab.matmul(a, b, False), lhsT)

"""Row kernels in the reference's kernel-level form (nkilab/kernels/norm.py).

x, out are [R, D]; the B200 kernels map one row to one warp instead of 128 rows to
the SBUF partitions, so P only documents the reference's tile height.
"""
from __future__ import annotations

import torch

from .. import _torch_ops  # noqa: F401
from .._host import like_input, to_device

P = 128  # reference row tile (SBUF partitions)


def softmax_unfused(x):
    """Three HBM round trips: max, exp + row sum (fp32), divide (norm.py:22-62)."""
    xd = to_device(x)
    return like_input(torch.ops.nkilab.softmax(xd, False), x)


def softmax_fused(x):
    """One pass: -max, exp with row sum, reciprocal, multiply (norm.py:65-89)."""
    xd = to_device(x)
    return like_input(torch.ops.nkilab.softmax(xd, True), x)


def rmsnorm_fused(x, weight, eps: float = 1e-6):
    """y = x * rsqrt(mean(x^2) + eps) * weight in one pass (norm.py:92-118)."""
    xd = to_device(x)
    wd = to_device(weight, xd.device).to(xd.dtype)
    return like_input(torch.ops.nkilab.rmsnorm(xd, wd, float(eps)), x)


def swiglu_fused(gate, up):
    """y = silu(gate) * up in one pass (norm.py:121-136)."""
    gd = to_device(gate)
    return like_input(torch.ops.nkilab.swiglu(gd, to_device(up, gd.device)), gate)

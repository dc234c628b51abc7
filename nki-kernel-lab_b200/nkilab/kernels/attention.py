"""Causal attention in the reference's kernel-level form (nkilab/kernels/attention.py).

Kernel layout, as prepared by the reference's ops.attention: qT, kT [H, d, S],
v [H, S, d], out [H, S, d], S a multiple of T. The B200 kernels read q and k as
[H, S, d], so qT / kT are transposed on the device first. All flash variants run
the same tcgen05 flash kernel; the reference's variants differ only in engine
scheduling and produce identical numerics (its tests/test_attention.py:67-70).
"""
from __future__ import annotations

import torch

from .. import _torch_ops  # noqa: F401
from .._host import like_input, to_device

T = 128  # query / key tile
NEG_INF = -3.0e38  # score of masked positions in the naive kernel


def _run(qT, kT, v, scale: float, naive: bool):
    H, d, S = qT.shape
    assert S % T == 0 and d <= 128
    q = to_device(qT).transpose(1, 2).contiguous()
    k = to_device(kT, q.device).transpose(1, 2).contiguous()
    vd = to_device(v, q.device)
    dp = d
    if q.dtype == torch.bfloat16 and not naive and d not in (64, 128):
        dp = 64 if d < 64 else 128
        q, k, vd = (torch.nn.functional.pad(t, (0, dp - d)) for t in (q, k, vd))
    o = torch.ops.nkilab.attention(q, k, vd, float(scale), naive)
    if dp != d:
        o = o[..., :d].contiguous()
    return like_input(o, v)


def attention_naive(qT, kT, v, scale: float):
    """Scores [H, S, S] fp32 and probabilities in HBM, then P @ V (attention.py:35-89)."""
    return _run(qT, kT, v, scale, True)


def flash_attention(qT, kT, v, scale: float):
    """Online-softmax flash attention with causal tile skipping (attention.py:155-176)."""
    return _run(qT, kT, v, scale, False)


def flash_attention_kv_resident(qT, kT, v, scale: float):
    """Same numerics as flash_attention (attention.py:179-201)."""
    return _run(qT, kT, v, scale, False)


def flash_attention_balanced(qT, kT, v, scale: float):
    """Same numerics as flash_attention (attention.py:249-277)."""
    return _run(qT, kT, v, scale, False)


def flash_attention_pipelined(qT, kT, v, scale: float, ILP: int = 2):
    """Same numerics as flash_attention (attention.py:280-325). ILP is accepted for
    signature parity; the B200 kernel overlaps tiles with its warp-specialised pipeline."""
    return _run(qT, kT, v, scale, False)

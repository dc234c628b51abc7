"""Host-side ops: the drop-in boundary of the reference's ``nkilab.ops``.

Same names, signatures, argument meaning and error behaviour as the reference
(nkilab/ops.py:1-91 in Nags-gk/nki-kernel-lab): every op takes NumPy arrays (float32
or ml_dtypes.bfloat16) and returns a new NumPy array of the input's dtype, accepts
any shape, and pads / crops internally. Where the reference runs an NKI kernel on
the CPU simulator, these run the B200 CUDA kernels of libnkilab_b200.so through the
``torch.ops.nkilab`` custom ops. They also accept torch tensors: a CUDA tensor stays
on the device (no copies), a CPU tensor (pinned or not) is copied in and the result
copied back to the CPU.

There is no CPU fallback: on a machine without a GPU every op raises.
"""
from __future__ import annotations

import math

import torch

from . import _torch_ops  # noqa: F401  (registers torch.ops.nkilab.*)
from ._host import dtype_of as _dtype_of
from ._host import like_input as _like_input
from ._host import to_device as _to_device
from .kernels import attention as _attn

__all__ = ["choose_blocks", "matmul", "softmax", "rmsnorm", "swiglu", "attention", "ATTENTION_VARIANTS"]


# --------------------------------------------------------------------------- matmul

def choose_blocks(m_tiles: int, n_tiles: int) -> tuple[int, int]:
    """Largest BM x BN output block (BM in {1,2,4}, BN in {1,2,4,8}, BM*BN <= 8) dividing
    the (m_tiles, n_tiles) grid; among equal areas the wider block wins.

    Same rule as nkilab/ops.py:27-35 (8 PSUM banks of [128, 512] fp32 per partition on
    Trainium2). The B200 GEMM does not need it -- its output tile lives in TMEM and is
    chosen by the kernel -- but kernels.matmul.matmul_blocked validates block
    arguments against the same budget.
    """
    cands = [(bm, bn) for bm in (1, 2, 4) for bn in (1, 2, 4, 8)
             if bm * bn <= 8 and m_tiles % bm == 0 and n_tiles % bn == 0]
    return max(cands, key=lambda c: (c[0] * c[1], c[1]))


def matmul(a, b, variant: str = "blocked"):
    """C = A @ B for any shapes, fp32 accumulation, output in A's dtype (ops.py:38-52).

    variant "blocked" (default) runs the TMA + tcgen05 GEMM (bf16) or the exact fp32
    CUDA-core GEMM (float32); "naive" runs the no-reuse kernel.
    """
    M, K = a.shape
    K2, N = b.shape
    assert K == K2, (a.shape, b.shape)
    if _dtype_of(a) != _dtype_of(b):
        raise TypeError(f"matmul operands differ in dtype: {_dtype_of(a)} vs {_dtype_of(b)}")
    ad = _to_device(a)
    bd = _to_device(b, ad.device)
    naive = variant == "naive"
    if ad.dtype == torch.bfloat16 and not naive and (K % 8 or N % 8):
        # TMA rows must be 16-byte multiples: zero-pad K and N to multiples of 8 (the
        # padded products are zeros), then crop, as the reference pads to its tiles.
        Kp, Np = -(-K // 8) * 8, -(-N // 8) * 8
        ad = torch.nn.functional.pad(ad, (0, Kp - K))
        bd = torch.nn.functional.pad(bd, (0, Np - N, 0, Kp - K))
        c = torch.ops.nkilab.matmul(ad, bd, False)[:, :N].contiguous()
    else:
        c = torch.ops.nkilab.matmul(ad, bd, naive)
    return _like_input(c, a)


# --------------------------------------------------------------------------- row kernels

def softmax(x, fused: bool = True):
    """Row softmax over the last dim (ops.py:55-57): fused single pass, or the 3-pass
    unfused kernel sequence when fused=False."""
    xd = _to_device(x)
    return _like_input(torch.ops.nkilab.softmax(xd, bool(fused)), x)


def rmsnorm(x, weight, eps: float = 1e-6):
    """y = x * rsqrt(mean(x^2) + eps) * weight over the last dim (ops.py:60-61)."""
    xd = _to_device(x)
    wd = _to_device(weight, xd.device)
    if wd.dtype != xd.dtype:
        wd = wd.to(xd.dtype)
    return _like_input(torch.ops.nkilab.rmsnorm(xd, wd, float(eps)), x)


def swiglu(gate, up):
    """y = silu(gate) * up elementwise (ops.py:64-65)."""
    gd = _to_device(gate)
    ud = _to_device(up, gd.device)
    return _like_input(torch.ops.nkilab.swiglu(gd, ud), gate)


# --------------------------------------------------------------------------- attention

ATTENTION_VARIANTS = {
    "naive": _attn.attention_naive,
    "flash": _attn.flash_attention,
    "flash_kv_resident": _attn.flash_attention_kv_resident,
    "flash_balanced": _attn.flash_attention_balanced,
    "flash_pipelined": _attn.flash_attention_pipelined,
}


def attention(q, k, v, variant: str = "flash_pipelined"):
    """Causal attention, q, k, v: [H, S, d], scale 1/sqrt(d) (ops.py:77-91).

    Any S: the kernels handle a partial last tile directly, so there is no host
    padding of the sequence. bf16 head dims other than 64/128 are zero-padded to the
    next of those (padding q/k columns adds zeros to every score; padded v columns
    are cropped). Every "flash*" variant runs the same tcgen05 flash kernel (the
    reference's variants share numerics, tests/test_attention.py:67-70);
    "naive" materialises the scores and probabilities.

    Extension beyond the reference: k and v may carry fewer heads than q (grouped-query
    or multi-query attention); query head h then uses key/value head h // (H // Hkv).
    """
    if variant not in ATTENTION_VARIANTS:
        raise KeyError(variant)
    H, S, d = q.shape
    assert d <= 128, f"head_dim {d} > 128"
    qd = _to_device(q)
    kd = _to_device(k, qd.device)
    vd = _to_device(v, qd.device)
    scale = 1.0 / math.sqrt(d)
    naive = variant == "naive"
    dp = d
    if qd.dtype == torch.bfloat16 and not naive and d not in (64, 128):
        dp = 64 if d < 64 else 128
        pad = (0, dp - d)
        qd, kd, vd = (torch.nn.functional.pad(t, pad) for t in (qd, kd, vd))
    o = torch.ops.nkilab.attention(qd, kd, vd, scale, naive)
    if dp != d:
        o = o[..., :d].contiguous()
    return _like_input(o, q)


def rope(x, base: float = 10000.0, pos_offset: int = 0):
    """Rotary position embedding, rotate-half convention, of x: [H, S, d] (extension
    beyond the reference, which lists rotary embeddings as not done, README.md:89).
    Position of row s is s + pos_offset; theta_i = base^(-2i/d). NumPy or torch in,
    same kind out."""
    xd = _to_device(x).contiguous()
    o = torch.ops.nkilab.rope(xd, float(base), int(pos_offset))
    return _like_input(o, x)

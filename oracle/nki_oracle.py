"""CPU restatement of the reference's kernel arithmetic (test infrastructure only).

THIS MODULE IS THE CHECKER, NOT THE PRODUCT. Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg may import it. Nothing under nki-kernel-lab_b200/ imports
it, and the product path never falls back to it.

Each function restates, in torch fp32 on the CPU, what one NKI kernel of
Nags-gk/nki-kernel-lab computes, instruction by instruction, with the reference's
rounding points (where a value is written to a tile of the input dtype it is rounded
here with round-to-nearest-even). Citations are path:line in the reference.

Pinning: tests/golden/ holds vectors produced by running the reference's own kernel
source (nkilab/kernels/*.py, nkilab/ops.py, nkilab/model.py) on a NumPy restatement
of the NKI instructions it calls (tests/golden/nki_shim.py); tests/test_oracle.py
checks this module against every one of them and against the reference tests' own
PyTorch references and known-answer checks.
"""
from __future__ import annotations

import math

import torch

T = 128            # attention tile, nkilab/kernels/attention.py:24
NEG_INF = -3.0e38  # nkilab/kernels/attention.py:25


def _f32(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.float32)


# --------------------------------------------------------------------------- row kernels

def softmax_fused(x: torch.Tensor) -> torch.Tensor:
    """nkilab/kernels/norm.py:65-89: neg_max = -max (:79), e = exp(x + neg_max) with
    the row sum in the same step (:82-83), rinv = 1/sum (:85), y = e * rinv (:87)."""
    xf = _f32(x)
    neg_max = -xf.amax(dim=-1, keepdim=True)
    e = torch.exp(xf + neg_max)
    ssum = e.sum(dim=-1, keepdim=True)
    rinv = 1.0 / ssum
    return (e * rinv).to(x.dtype)


def softmax_unfused(x: torch.Tensor) -> torch.Tensor:
    """nkilab/kernels/norm.py:22-62: m = max (:39), e = exp(x - m) (:47-49),
    s = sum e (:51), y = e / s (:60)."""
    xf = _f32(x)
    m = xf.amax(dim=-1, keepdim=True)
    e = torch.exp(xf - m)
    s = e.sum(dim=-1, keepdim=True)
    return (e / s).to(x.dtype)


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, acc: torch.dtype = torch.float32) -> torch.Tensor:
    """nkilab/kernels/norm.py:92-118: ssq = sum(x^2) fp32 (:107-108),
    ms = ssq * (1/D) + eps (:110), rstd = rsqrt(ms) (:112), xn = x * rstd fp32 (:114),
    y = xn * weight rounded to x.dtype (:116). `acc` (float32 as the reference, or
    float64 for an error floor) is the precision of every intermediate."""
    D = x.shape[-1]
    xf = x.to(acc)
    ssq = (xf * xf).sum(dim=-1, keepdim=True)
    ms = ssq * torch.tensor(1.0 / D, dtype=acc) + torch.tensor(eps, dtype=acc)
    rstd = torch.rsqrt(ms)
    xn = xf * rstd
    return (xn * weight.to(x.dtype).to(acc)).to(x.dtype)


def swiglu(gate: torch.Tensor, up: torch.Tensor, acc: torch.dtype = torch.float32) -> torch.Tensor:
    """nkilab/kernels/norm.py:121-136: a = silu(gate) fp32 (:131-132), y = a * up
    rounded to gate.dtype (:133-134)."""
    g = gate.to(acc)
    a = g / (1.0 + torch.exp(-g))
    return (a * up.to(acc)).to(gate.dtype)


# --------------------------------------------------------------------------- matmul

def matmul(a: torch.Tensor, b: torch.Tensor, acc: torch.dtype = torch.float32) -> torch.Tensor:
    """nkilab/kernels/matmul.py:46-82 (and :24-43): fp32 accumulation of exact products
    (PSUM, :62-75), one rounding to lhsT.dtype = a.dtype on the copy out (:76-79)."""
    return (a.to(acc) @ b.to(acc)).to(a.dtype)


def choose_blocks(m_tiles: int, n_tiles: int) -> tuple[int, int]:
    """nkilab/ops.py:27-35: largest BM*BN <= 8 dividing the grid, ties -> larger BN."""
    best = None
    for bm in (1, 2, 4):
        for bn in (1, 2, 4, 8):
            if bm * bn > 8 or m_tiles % bm or n_tiles % bn:
                continue
            key = (bm * bn, bn)
            if best is None or key > best[0]:
                best = (key, (bm, bn))
    return best[1]


# --------------------------------------------------------------------------- attention

def _pad_seq(t: torch.Tensor, Sp: int) -> torch.Tensor:
    H, S, d = t.shape
    if S == Sp:
        return t
    out = torch.zeros((H, Sp, d), dtype=t.dtype)
    out[:, :S] = t
    return out


def attention_flash(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None,
                    acc: torch.dtype = torch.float32) -> torch.Tensor:
    """Causal flash attention as nkilab/kernels/attention.py:280-325 with the balanced
    update :204-246 (the default "flash_pipelined" variant), batched over heads.

    Host side as nkilab/ops.py:77-91: S padded to a multiple of 128 at the end
    (:83-87), scale 1/sqrt(d) (:90), output cropped (:91). Per 128-query tile i:
      nm = +3e38, l = 0, o = 0 (:305-310)
      for key tile j <= i (:312-315):
        s = q_i k_j^T fp32 (:318); diagonal tile masked to -3e38 where q < k (:216-221)
        nm' = min(rowmax(s) * -scale, nm) (:224-227)
        e = exp(s * scale + nm') fp32, rsum = sum e, p = e rounded to v.dtype (:228-231)
        corr = exp(-nm + nm') (:232-233); l = l * corr + rsum (:234-236)
        o = o * corr + p @ v_j (fp32 accumulate) (:237-245)
      out_i = o * (1/l) rounded to v.dtype (:137-142)
    `acc` is the precision of scores, statistics and accumulators (float32 as the
    reference; float64 gives an error floor with the same bf16 rounding points).
    """
    H, S, d = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    dt = v.dtype
    nt = -(-S // T)
    Sp = nt * T
    qf, kf, vf = (_pad_seq(t, Sp).to(acc) for t in (q, k, v))
    out = torch.empty((H, Sp, d), dtype=dt)
    sc = torch.tensor(scale, dtype=acc)
    rows = torch.arange(T).view(T, 1)
    cols = torch.arange(T).view(1, T)
    diag_keep = (rows - cols) >= 0
    for i in range(nt):
        qi = qf[:, i * T:(i + 1) * T]
        nm = torch.full((H, T, 1), -NEG_INF, dtype=acc)
        l = torch.zeros((H, T, 1), dtype=acc)
        o = torch.zeros((H, T, d), dtype=acc)
        for j in range(i + 1):
            s = qi @ kf[:, j * T:(j + 1) * T].transpose(1, 2)
            if j == i:
                s = torch.where(diag_keep, s, torch.tensor(NEG_INF, dtype=acc))
            tmax = s.amax(dim=-1, keepdim=True)
            nm_new = torch.minimum(tmax * (-sc), nm)
            e = torch.exp(s * sc + nm_new)
            rsum = e.sum(dim=-1, keepdim=True)
            p = e.to(dt)
            corr = torch.exp(nm * -1.0 + nm_new)
            l = l * corr + rsum
            pv = p.to(acc) @ vf[:, j * T:(j + 1) * T]
            o = o * corr + pv
            nm = nm_new
        linv = 1.0 / l
        out[:, i * T:(i + 1) * T] = (o * linv).to(dt)
    return out[:, :S].contiguous()


def attention_naive(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None) -> torch.Tensor:
    """nkilab/kernels/attention.py:35-89: scores = (q k^T) * scale masked to -3e38
    where q < k, fp32 in HBM (:44-57); per row nmax = -max, e = exp(row + nmax),
    rinv = 1/sum, p = e * rinv rounded to v.dtype (:58-72); out = p @ v fp32
    accumulate, rounded to v.dtype (:73-88). Host padding as attention_flash."""
    H, S, d = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    dt = v.dtype
    Sp = -(-S // T) * T
    qf, kf, vf = (_f32(_pad_seq(t, Sp)) for t in (q, k, v))
    s = (qf @ kf.transpose(1, 2)) * torch.tensor(scale, dtype=torch.float32)
    idx = torch.arange(Sp)
    keep = (idx.view(Sp, 1) - idx.view(1, Sp)) >= 0
    s = torch.where(keep, s, torch.tensor(NEG_INF, dtype=torch.float32))
    nmax = -s.amax(dim=-1, keepdim=True)
    e = torch.exp(s + nmax)
    rinv = 1.0 / e.sum(dim=-1, keepdim=True)
    p = (e * rinv).to(dt)
    out = (_f32(p) @ vf).to(dt)
    return out[:, :S].contiguous()


# --------------------------------------------------------------------------- decoder block

def decoder_block(x: torch.Tensor, norm1: torch.Tensor, wqkv: torch.Tensor, wo: torch.Tensor, norm2: torch.Tensor,
                  wg: torch.Tensor, wu: torch.Tensor, wd: torch.Tensor, n_heads: int, eps: float = 1e-6,
                  naive_attention: bool = False, acc: torch.dtype = torch.float32) -> torch.Tensor:
    """nkilab/model.py:70-89 (nki_forward) for x [S, d]: weights are given in
    nn.Linear layout [out, in] and used transposed in x's dtype (:76-77); residual adds
    in x.dtype (:86, :89). `acc` as in attention_flash: float64 keeps every bf16
    rounding point of the block and removes the fp32 accumulation error, so the
    distance between the float32 and float64 results is the floor two correct fp32
    implementations of the block can be expected to differ by."""
    S, d = x.shape
    hd = d // n_heads
    dt = x.dtype

    def w(m: torch.Tensor) -> torch.Tensor:
        return m.t().contiguous().to(dt)

    h = rmsnorm(x, norm1.to(dt), eps, acc)
    qkv = matmul(h, w(wqkv), acc)
    q, k, v = (qkv[:, i * d:(i + 1) * d].reshape(S, n_heads, hd).transpose(0, 1).contiguous() for i in range(3))
    a = attention_naive(q, k, v) if naive_attention else attention_flash(q, k, v, acc=acc)
    x = (x.to(acc) + matmul(a.transpose(0, 1).reshape(S, d), w(wo), acc).to(acc)).to(dt)
    h = rmsnorm(x, norm2.to(dt), eps, acc)
    act = swiglu(matmul(h, w(wg), acc), matmul(h, w(wu), acc), acc)
    return (x.to(acc) + matmul(act, w(wd), acc).to(acc)).to(dt)

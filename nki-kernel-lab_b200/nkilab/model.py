"""Llama-style decoder block, run two ways: PyTorch eager and the B200 kernels.

    x = x + Wo . causal_attention(split_heads(RMSNorm(x) . Wqkv))
    x = x + Wd . (silu(RMSNorm(x) . Wg) * (RMSNorm(x) . Wu))

Same API as the reference's nkilab/model.py (BlockConfig, RMSNorm, DecoderBlock,
nki_forward; Nags-gk/nki-kernel-lab nkilab/model.py:1-89). DecoderBlock builds its
submodules in the reference's order and re-initialises the norm weights the same
way, so a given torch seed yields the same weights as the reference block.

``nki_forward`` runs every matmul, RMSNorm, attention and SwiGLU through nkilab.ops
(the CUDA kernels). With NumPy input it behaves like the reference (weights taken
from the block and cast to x's dtype, result returned as NumPy). With a CUDA tensor
input everything stays on the device, the transposed weights are cached on the block
per (dtype, device) and refreshed when a parameter changes, and x may carry a leading
batch dimension ([B, S, d]): the GEMMs and row kernels then run over all B*S rows and
attention over all B*H heads. Rotary embeddings are left out, as in the reference.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _torch_ops, ops


@dataclass
class BlockConfig:
    d_model: int = 256
    n_heads: int = 4
    d_ff: int = 1024
    eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads


class RMSNorm(nn.Module):
    def __init__(self, d: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d))

    def forward(self, x):
        ms = x.pow(2).mean(-1, keepdim=True)
        return x * torch.rsqrt(ms + self.eps) * self.weight


class DecoderBlock(nn.Module):
    """PyTorch reference block; x: [S, d]."""

    def __init__(self, cfg: BlockConfig):
        super().__init__()
        self.cfg = cfg
        d, f = cfg.d_model, cfg.d_ff
        # creation order fixes which random numbers each weight receives
        self.norm1 = RMSNorm(d, cfg.eps)
        self.norm2 = RMSNorm(d, cfg.eps)
        self.wqkv = nn.Linear(d, 3 * d, bias=False)
        self.wo = nn.Linear(d, d, bias=False)
        self.wg = nn.Linear(d, f, bias=False)
        self.wu = nn.Linear(d, f, bias=False)
        self.wd = nn.Linear(f, d, bias=False)
        with torch.no_grad():  # non-trivial norm gains, as in the reference
            for norm in (self.norm1, self.norm2):
                norm.weight.uniform_(0.5, 1.5)

    def forward(self, x):
        S, d = x.shape
        H, hd = self.cfg.n_heads, self.cfg.head_dim
        qkv = self.wqkv(self.norm1(x))
        q, k, v = (t.reshape(S, H, hd).transpose(0, 1) for t in qkv.split(d, dim=-1))
        attn = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.wo(attn.transpose(0, 1).reshape(S, d))
        h = self.norm2(x)
        return x + self.wd(F.silu(self.wg(h)) * self.wu(h))


_WEIGHT_NAMES = ("wqkv", "wo", "wg", "wu", "wd")


def device_weights(block: DecoderBlock, dtype: torch.dtype, device) -> dict:
    """Transposed ([in, out]) weights and norm gains of `block` on `device` in `dtype`,
    cached on the block; the cache is rebuilt when any parameter is modified."""
    stamp = tuple((p.data_ptr(), p._version) for p in block.parameters())
    key = (dtype, str(device))
    cache = block.__dict__.setdefault("_nkl_weight_cache", {})
    hit = cache.get(key)
    if hit is not None and hit[0] == stamp:
        return hit[1]
    with torch.no_grad():
        w = {n: getattr(block, n).weight.detach().t().to(device=device, dtype=dtype).contiguous() for n in _WEIGHT_NAMES}
        w["norm1"] = block.norm1.weight.detach().to(device=device, dtype=dtype).contiguous()
        w["norm2"] = block.norm2.weight.detach().to(device=device, dtype=dtype).contiguous()
        if dtype == torch.bfloat16 and w["wg"].shape[1] % _torch_ops.SWIGLU_BLOCK == 0:
            # one GEMM for gate and up with SwiGLU in its epilogue (bit-identical to the
            # unfused matmul -> matmul -> swiglu path)
            w["wgu"] = _torch_ops.interleave_gate_up(w["wg"], w["wu"])
    cache[key] = (stamp, w)
    return w


def _forward_device(block: DecoderBlock, x: torch.Tensor, attention_variant: str) -> torch.Tensor:
    cfg = block.cfg
    d, H, hd = cfg.d_model, cfg.n_heads, cfg.head_dim
    lead = x.shape[:-1]
    S = x.shape[-2]
    B = x[..., 0, 0].numel() if x.dim() == 3 else 1
    w = device_weights(block, x.dtype, x.device)
    x2 = x.reshape(-1, d)
    h = ops.rmsnorm(x2, w["norm1"], cfg.eps)
    qkv = ops.matmul(h, w["wqkv"]).view(B, S, 3, H, hd)
    if attention_variant != "naive" and x.dtype == torch.bfloat16 and hd in (64, 128):
        # q, k, v read straight out of the fused projection and the output written in the
        # [B*S, d] layout the Wo GEMM reads: strided views, no transposing copies
        a = torch.empty(B, S, H, hd, dtype=x.dtype, device=x.device)
        for b in range(B):
            q, k, v = (qkv[b, :, i].transpose(0, 1) for i in range(3))
            torch.ops.nkilab.attention_strided_(q, k, v, a[b].transpose(0, 1), 1.0 / math.sqrt(hd))
        a = a.view(B * S, d)
    else:
        q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3).reshape(B * H, S, hd) for i in range(3))
        a = ops.attention(q, k, v, variant=attention_variant)
        a = a.view(B, H, S, hd).permute(0, 2, 1, 3).reshape(B * S, d)
    # residual add fused with the second RMSNorm (same rounding as add-then-norm)
    x2, h = torch.ops.nkilab.add_rmsnorm(x2.contiguous(), ops.matmul(a, w["wo"]).contiguous(), w["norm2"], cfg.eps)
    if "wgu" in w:
        act = torch.ops.nkilab.matmul_swiglu(h.contiguous(), w["wgu"])
    else:
        act = ops.swiglu(ops.matmul(h, w["wg"]), ops.matmul(h, w["wu"]))
    if x.dtype == torch.bfloat16:  # residual add in the down projection's epilogue (same bits)
        out = torch.ops.nkilab.matmul_residual(act.contiguous(), w["wd"], x2.contiguous())
    else:
        out = x2 + ops.matmul(act, w["wd"])
    return out.view(*lead, d)


def nki_forward(block: DecoderBlock, x, attention_variant: str = "flash_pipelined"):
    """The same block with every heavy op on the B200 kernels (nkilab/model.py:70-89)."""
    if isinstance(x, torch.Tensor) and x.device.type == "cuda":
        return _forward_device(block, x, attention_variant)
    cfg = block.cfg
    S, d = x.shape
    H, hd = cfg.n_heads, cfg.head_dim

    def w(lin: nn.Linear) -> np.ndarray:  # nn.Linear holds [out, in]; the product needs [in, out]
        return lin.weight.detach().numpy().T.astype(x.dtype).copy()

    def g(norm: RMSNorm) -> np.ndarray:
        return norm.weight.detach().numpy().astype(x.dtype)

    h = ops.rmsnorm(x, g(block.norm1), cfg.eps)
    qkv = ops.matmul(h, w(block.wqkv))
    q, k, v = (np.ascontiguousarray(qkv[:, i * d:(i + 1) * d].reshape(S, H, hd).transpose(1, 0, 2)) for i in range(3))
    a = ops.attention(q, k, v, variant=attention_variant)
    x = x + ops.matmul(np.ascontiguousarray(a.transpose(1, 0, 2).reshape(S, d)), w(block.wo))
    h = ops.rmsnorm(x, g(block.norm2), cfg.eps)
    act = ops.swiglu(ops.matmul(h, w(block.wg)), ops.matmul(h, w(block.wu)))
    return x + ops.matmul(act, w(block.wd))

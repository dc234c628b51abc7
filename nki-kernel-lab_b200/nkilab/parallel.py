"""Multi-GPU execution of the kernel set: one process per GPU, torch.distributed
(NCCL over NVLink / NVSwitch on the GPU box) for the collectives.

The reference runs on a single NeuronCore and has no distributed code; this module
adds the sharding of the B200 build's north star:

* attention   heads are independent: rank r computes heads [h0, h1) of its share,
              then one all-gather assembles the [H, S, d] output on every rank.
* row kernels rows are independent: rank r runs RMSNorm / softmax / SwiGLU on its
              row block, then one all-gather assembles the output.
* decoder     tensor parallel over heads and FFN columns with sequence-parallel
  block       row shards (Megatron style): RMSNorm and the residual adds run on the
              local rows; all-gather before the QKV and gate/up GEMMs; each rank
              holds the Wqkv columns of its heads, the Wo rows of its heads, the
              Wg/Wu columns and the Wd rows of its FFN slice; reduce-scatter after
              Wo and after Wd; a final all-gather returns the full block output.
              The exact block needs the two reduce-scatters: a partial sum over
              heads (Wo) or FFN columns (Wd) is not a gather.

Shards are as even as possible (sizes differ by at most one unit); collectives pad
to the largest shard and crop. Every rank issues the same collectives in the same
order. The per-shard compute is the CUDA ops by default; `compute` arguments exist
so the host-side logic can be exercised with gloo ranks on CPU in tests.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional, Sequence

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's share of n units; the first n % world ranks get one more."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _world(group) -> tuple[int, int]:
    if group is None and not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def all_gather_dim0(local: torch.Tensor, n_total: int, group=None) -> torch.Tensor:
    """Concatenate every rank's dim-0 shard (shard_range layout) into n_total rows."""
    world, rank = _world(group)
    if world == 1:
        return local
    sizes = [shard_range(n_total, world, r) for r in range(world)]
    max_rows = max(e - s for s, e in sizes)
    if local.shape[0] != max_rows:
        pad = torch.zeros((max_rows - local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        local = torch.cat([local, pad], 0)
    out = torch.empty((world * max_rows,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    parts = [out[r * max_rows:r * max_rows + (e - s)] for r, (s, e) in enumerate(sizes)]
    return torch.cat(parts, 0)


def reduce_scatter_dim0(full: torch.Tensor, group=None) -> torch.Tensor:
    """Sum `full` over ranks and return this rank's dim-0 shard (shard_range layout).
    The sum is taken in fp32 for bf16 inputs and rounded once."""
    world, rank = _world(group)
    if world == 1:
        return full
    n = full.shape[0]
    sizes = [shard_range(n, world, r) for r in range(world)]
    max_rows = max(e - s for s, e in sizes)
    acc = full.float() if full.dtype == torch.bfloat16 else full
    chunks = []
    for s, e in sizes:
        c = acc[s:e]
        if e - s != max_rows:
            c = torch.cat([c, torch.zeros((max_rows - (e - s),) + tuple(acc.shape[1:]), dtype=acc.dtype,
                                          device=acc.device)], 0)
        chunks.append(c)
    inp = torch.cat(chunks, 0).contiguous()
    out = torch.empty((max_rows,) + tuple(acc.shape[1:]), dtype=acc.dtype, device=acc.device)
    dist.reduce_scatter_tensor(out, inp, op=dist.ReduceOp.SUM, group=group)
    s, e = sizes[rank]
    return out[:e - s].to(full.dtype)


# --------------------------------------------------------------------------- attention / rows

def _default_attention(q, k, v, variant):
    from . import ops

    return ops.attention(q, k, v, variant=variant)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, variant: str = "flash_pipelined", group=None,
              compute: Optional[Callable] = None) -> torch.Tensor:
    """Head-sharded causal attention. q, k, v: [H, S, d], the same full tensors on
    every rank (or only this rank's head rows are read). Returns the full [H, S, d]
    output on every rank after one all-gather."""
    world, rank = _world(group)
    H = q.shape[0]
    h0, h1 = shard_range(H, world, rank)
    fn = compute or _default_attention
    local = fn(q[h0:h1].contiguous(), k[h0:h1].contiguous(), v[h0:h1].contiguous(), variant)
    return all_gather_dim0(local, H, group)


def row_op(op: str, *tensors: torch.Tensor, group=None, compute: Optional[Callable] = None, **kw) -> torch.Tensor:
    """Row-sharded row kernel: op in {"rmsnorm", "softmax", "swiglu"}. Row tensors
    ([R, D], full on every rank) are split by rows; a 1-D rmsnorm weight is passed
    whole. Returns the full [R, D] output on every rank."""
    world, rank = _world(group)
    R = tensors[0].shape[0]
    r0, r1 = shard_range(R, world, rank)
    args = [t[r0:r1].contiguous() if t.dim() > 1 else t for t in tensors]
    if compute is not None:
        local = compute(op, *args, **kw)
    else:
        from . import ops

        local = getattr(ops, op)(*args, **kw)
    return all_gather_dim0(local, R, group)


def matmul(a: torch.Tensor, b: torch.Tensor, group=None, compute: Optional[Callable] = None,
           block: int = 128) -> torch.Tensor:
    """Column-sharded GEMM: c = a @ b with b's columns split over the ranks in units of
    `block` columns (so every local bf16 GEMM keeps N a multiple of 8); each rank multiplies
    the full a by its column block of b, then one all-gather assembles the full [M, N]
    c on every rank. a: [M, K], b: [K, N], the same full tensors on every rank."""
    world, rank = _world(group)
    N = b.shape[1]
    units = (N + block - 1) // block
    u0, u1 = shard_range(units, world, rank)
    c0, c1 = min(u0 * block, N), min(u1 * block, N)
    if compute is None:
        from . import ops

        compute = ops.matmul
    if c1 > c0:
        local = compute(a, b[:, c0:c1].contiguous())
    else:
        local = torch.zeros((a.shape[0], 0), dtype=a.dtype, device=a.device)
    if world == 1:
        return local
    # gather the column blocks as row blocks of c^T (all_gather_dim0 shards dim 0)
    sizes = [shard_range(units, world, r) for r in range(world)]
    widths = [min(e * block, N) - min(s * block, N) for s, e in sizes]
    max_w = max(widths)
    lt = local.t().contiguous()
    if lt.shape[0] != max_w:
        lt = torch.cat([lt, torch.zeros((max_w - lt.shape[0], lt.shape[1]), dtype=lt.dtype, device=lt.device)], 0)
    out = torch.empty((world * max_w, lt.shape[1]), dtype=lt.dtype, device=lt.device)
    dist.all_gather_into_tensor(out, lt, group=group)
    return torch.cat([out[r * max_w:r * max_w + widths[r]] for r in range(world)], 0).t().contiguous()


# --------------------------------------------------------------------------- decoder block

@dataclass
class ShardedBlockWeights:
    """This rank's slice of a DecoderBlock, transposed to [in, out] for x @ W."""
    norm1: torch.Tensor
    norm2: torch.Tensor
    wqkv: torch.Tensor   # [d, 3 * local_heads * hd]: q | k | v columns of the local heads
    wo: torch.Tensor     # [local_heads * hd, d]: rows of Wo^T for the local heads
    wg: torch.Tensor     # [d, local_ff]
    wu: torch.Tensor     # [d, local_ff]
    wd: torch.Tensor     # [local_ff, d]
    heads: tuple[int, int]
    ff: tuple[int, int]


def shard_block(block, world: int, rank: int, dtype: torch.dtype, device) -> ShardedBlockWeights:
    cfg = block.cfg
    d, H, hd = cfg.d_model, cfg.n_heads, cfg.head_dim
    h0, h1 = shard_range(H, world, rank)
    f0, f1 = shard_range(cfg.d_ff, world, rank)
    with torch.no_grad():
        wqkv = block.wqkv.weight.detach()  # [3d, d]: q rows, then k, then v
        cols = [wqkv[i * d + h0 * hd:i * d + h1 * hd] for i in range(3)]

        def t(w):
            return w.t().contiguous().to(device=device, dtype=dtype)

        return ShardedBlockWeights(
            norm1=block.norm1.weight.detach().to(device=device, dtype=dtype),
            norm2=block.norm2.weight.detach().to(device=device, dtype=dtype),
            wqkv=t(torch.cat(cols, 0)),
            wo=t(block.wo.weight.detach()[:, h0 * hd:h1 * hd]),
            wg=t(block.wg.weight.detach()[f0:f1]),
            wu=t(block.wu.weight.detach()[f0:f1]),
            wd=t(block.wd.weight.detach()[:, f0:f1]),
            heads=(h0, h1), ff=(f0, f1))



def _device_ops():
    from . import ops

    return ops

def decoder_block(block, x: torch.Tensor, weights: Optional[ShardedBlockWeights] = None,
                  variant: str = "flash_pipelined", group=None, ops_module=None) -> torch.Tensor:
    """Tensor-parallel DecoderBlock forward. x: [S, d] full input on every rank.
    Returns the full [S, d] output on every rank."""
    world, rank = _world(group)
    if ops_module is None:
        from . import ops as ops_module
    cfg = block.cfg
    S, d = x.shape
    hd = cfg.head_dim
    w = weights or shard_block(block, world, rank, x.dtype, x.device)
    nh = w.heads[1] - w.heads[0]
    r0, r1 = shard_range(S, world, rank)
    x_loc = x[r0:r1]
    # attention half: norm on local rows -> gather rows -> local heads -> partial Wo -> reduce-scatter
    h = all_gather_dim0(ops_module.rmsnorm(x_loc.contiguous(), w.norm1, cfg.eps), S, group)
    if nh > 0:
        qkv = ops_module.matmul(h, w.wqkv)
        if (ops_module is _device_ops() and qkv.is_cuda and qkv.dtype == torch.bfloat16 and variant != "naive"
                and hd in (64, 128)):
            # local heads read straight out of the projection, output in the Wo layout
            a = torch.empty(S, nh, hd, dtype=qkv.dtype, device=qkv.device)
            q, k, v = (qkv[:, i * nh * hd:(i + 1) * nh * hd].view(S, nh, hd).transpose(0, 1) for i in range(3))
            torch.ops.nkilab.attention_strided_(q, k, v, a.transpose(0, 1), 1.0 / math.sqrt(hd))
            part = ops_module.matmul(a.view(S, nh * hd), w.wo)
        else:
            q, k, v = (qkv[:, i * nh * hd:(i + 1) * nh * hd].reshape(S, nh, hd).transpose(0, 1).contiguous()
                       for i in range(3))
            a = ops_module.attention(q, k, v, variant=variant)
            part = ops_module.matmul(a.transpose(0, 1).reshape(S, nh * hd).contiguous(), w.wo)
    else:
        part = torch.zeros((S, d), dtype=x.dtype, device=x.device)
    x_loc = (x_loc.float() + reduce_scatter_dim0(part, group).float()).to(x.dtype)
    # MLP half: norm on local rows -> gather rows -> local FFN columns -> partial Wd -> reduce-scatter
    h = all_gather_dim0(ops_module.rmsnorm(x_loc.contiguous(), w.norm2, cfg.eps), S, group)
    if w.ff[1] > w.ff[0]:
        act = ops_module.swiglu(ops_module.matmul(h, w.wg), ops_module.matmul(h, w.wu))
        part = ops_module.matmul(act, w.wd)
    else:
        part = torch.zeros((S, d), dtype=x.dtype, device=x.device)
    x_loc = (x_loc.float() + reduce_scatter_dim0(part, group).float()).to(x.dtype)
    return all_gather_dim0(x_loc, S, group)

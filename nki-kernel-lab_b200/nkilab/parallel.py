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

import ctypes
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
    if n_total % world == 0:  # even shards: gather straight into the result
        out = torch.empty((n_total,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
        return out
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
    if n % world == 0:  # even shards: scatter straight from the input
        out = torch.empty((n // world,) + tuple(acc.shape[1:]), dtype=acc.dtype, device=acc.device)
        dist.reduce_scatter_tensor(out, acc.contiguous(), op=dist.ReduceOp.SUM, group=group)
        return out.to(full.dtype)
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
    every rank (only this rank's head rows are read). Returns the full [H, S, d]
    output on every rank after one all-gather. With the default compute, q, k, v may
    be CPU tensors (pinned for asynchronous copies): only this rank's heads are copied
    to the current GPU, and the gathered output comes back on the CPU, as
    nkilab.ops.attention returns host input's result on the host."""
    world, rank = _world(group)
    H = q.shape[0]
    h0, h1 = shard_range(H, world, rank)
    if compute is None and q.device.type == "cpu":
        from ._host import like_input, to_device

        local = _default_attention(*(to_device(t[h0:h1]) for t in (q, k, v)), variant)
        return like_input(all_gather_dim0(local, H, group), q)
    fn = compute or _default_attention
    local = fn(q[h0:h1].contiguous(), k[h0:h1].contiguous(), v[h0:h1].contiguous(), variant)
    return all_gather_dim0(local, H, group)


def preferred_gather(world: int) -> str:
    """How the head-sharded attention's output should reach every rank: "nvlink" (the
    attention kernels store each output tile into every rank's buffer, PeerAttention) or
    "nccl" (an all-gather after the kernels). Measured on B200s with 8 heads x 2048 x 128,
    per step over NVLink against NCCL: two GPUs 31.4 against 43.4 us, four 37.9 against
    41.9 us, eight 48.1 against 44.2 us (with one head per rank most output tiles come from
    the split-KV combine kernel, whose stores to seven peers dominate)."""
    return "nvlink" if world <= 4 else "nccl"


class _RawCuda:
    """A device allocation seen through __cuda_array_interface__, so torch.as_tensor can
    view it without a copy (as uint16; the caller views it as bfloat16)."""

    def __init__(self, ptr: int, shape: tuple):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": "<u2", "data": (ptr, False), "version": 3,
                                         "strides": None}


class PeerAttention:
    """Head-sharded causal attention whose output gather runs over NVLink inside the
    attention launch (nkl_attention_allgather): every rank's attention kernel stores its
    finished output tiles into every rank's output buffer (CUDA IPC mappings of one
    buffer per rank), then a one-warp kernel exchanges per-call counts, so no library
    collective is involved. This is the B200 form of parallel.attention's
    compute-then-all-gather (which uses NCCL).

    Buffers: two output sets of [heads_total, seq, head_dim] bf16 per rank (consecutive
    calls alternate, so a rank never writes into a buffer a peer may still be reading) and
    one flag array, allocated once, their IPC handles exchanged with all_gather_object.
    __call__(q, k, v) takes this rank's heads (shard_range(heads_total, world, rank)) as
    contiguous bf16 CUDA tensors [local_heads, seq, head_dim] and returns this rank's full
    output buffer; it stays valid until the call after next (copy it to keep it longer).
    Every rank must make the same calls in the same order. close() (collective) releases
    the buffers."""

    def __init__(self, heads_total: int, seq: int, head_dim: int, group=None, device=None):
        from . import _native as N

        self.world, self.rank = _world(group)
        self.group = group
        self.heads_total, self.seq, self.head_dim = heads_total, seq, head_dim
        self.h0, self.h1 = shard_range(heads_total, self.world, self.rank)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        hb = int(N.lib.nkl_ipc_handle_bytes())
        self._own, self._opened = [], []
        nbytes = heads_total * seq * head_dim * 2
        handles = []
        with torch.cuda.device(self.device):
            for size in (nbytes, nbytes, 256):  # output set 0, output set 1, flags (world + 1 words)
                ptr, h = ctypes.c_void_p(), ctypes.create_string_buffer(hb)
                N.call("nkl_ipc_alloc", size, ctypes.byref(ptr), h)
                self._own.append(ptr.value)
                handles.append(h.raw)
            if self.world > 1:
                every = [None] * self.world
                dist.all_gather_object(every, handles, group=group)
            else:
                every = [handles]
            ptrs = []  # ptrs[r] = (out0, out1, flags) of rank r, valid on this device
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(tuple(self._own))
                    continue
                opened = []
                for h in every[r]:
                    p = ctypes.c_void_p()
                    N.call("nkl_ipc_open", ctypes.create_string_buffer(h, hb), ctypes.byref(p))
                    opened.append(p.value)
                    self._opened.append(p.value)
                ptrs.append(tuple(opened))
        arr = ctypes.c_void_p * self.world
        self._outs = [arr(*[ptrs[r][i] for r in range(self.world)]) for i in (0, 1)]
        self._flags = arr(*[ptrs[r][2] for r in range(self.world)])
        shape = (heads_total, seq, head_dim)
        self._views = [torch.as_tensor(_RawCuda(self._own[i], shape), device=self.device).view(torch.bfloat16)
                       for i in (0, 1)]
        self._calls = 0
        self.scale = 1.0 / math.sqrt(head_dim)

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        from . import _native as N
        from . import _torch_ops

        hl = self.h1 - self.h0
        want = (hl, self.seq, self.head_dim)
        for t in (q, k, v):
            if t.shape != want or t.dtype != torch.bfloat16 or not t.is_contiguous() or t.device != self.device:
                raise ValueError(f"PeerAttention: q, k, v must be contiguous bf16 {want} on {self.device}")
        which = self._calls & 1
        self._calls += 1
        st = torch.cuda.current_stream(self.device).cuda_stream
        with torch.cuda.device(self.device):
            nbytes = N.lib.nkl_attention_workspace_size(hl, self.seq, self.head_dim, N.BFLOAT16)
            ws = _torch_ops._attention_workspace(self.device, st, nbytes) if nbytes else None
            N.call("nkl_attention_allgather", q.data_ptr(), k.data_ptr(), v.data_ptr(), self._outs[which], self._flags,
                   self.world, self.rank, self.heads_total, self.h0, ws.data_ptr() if ws is not None else None, nbytes,
                   hl, self.seq, self.head_dim, self.scale, N.BFLOAT16, st)
        return self._views[which]

    def close(self) -> None:
        """Collective: every rank waits for the others, then releases its mappings and frees
        its buffers."""
        from . import _native as N

        if not self._own:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                N.call("nkl_ipc_close", ctypes.c_void_p(p))
            if self.world > 1:
                dist.barrier(group=self.group)
            for p in self._own:
                N.call("nkl_ipc_free", ctypes.c_void_p(p))
        self._own, self._opened, self._views = [], [], []


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

FF_UNIT = 128  # FFN columns are sharded in units of 128 (the fused SwiGLU GEMM's column block)


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
    wgu: Optional[torch.Tensor] = None  # [d, 2 * local_ff] gate/up interleaved for the fused SwiGLU GEMM


def ff_range(d_ff: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's FFN columns: whole 128-column units, as even as possible."""
    units = (d_ff + FF_UNIT - 1) // FF_UNIT
    u0, u1 = shard_range(units, world, rank)
    return min(u0 * FF_UNIT, d_ff), min(u1 * FF_UNIT, d_ff)


def shard_block(block, world: int, rank: int, dtype: torch.dtype, device) -> ShardedBlockWeights:
    """Slice `block`'s weights for `rank` of `world`: heads by shard_range, FFN columns by
    ff_range. The weights may live on any device; the slices are moved to `device`."""
    cfg = block.cfg
    d, H, hd = cfg.d_model, cfg.n_heads, cfg.head_dim
    h0, h1 = shard_range(H, world, rank)
    f0, f1 = ff_range(cfg.d_ff, world, rank)
    with torch.no_grad():
        wqkv = block.wqkv.weight.detach()  # [3d, d]: q rows, then k, then v
        cols = [wqkv[i * d + h0 * hd:i * d + h1 * hd] for i in range(3)]

        def t(w):
            return w.t().to(device=device, dtype=dtype).contiguous()

        sw = ShardedBlockWeights(
            norm1=block.norm1.weight.detach().to(device=device, dtype=dtype).contiguous(),
            norm2=block.norm2.weight.detach().to(device=device, dtype=dtype).contiguous(),
            wqkv=t(torch.cat(cols, 0)),
            wo=t(block.wo.weight.detach()[:, h0 * hd:h1 * hd]),
            wg=t(block.wg.weight.detach()[f0:f1]),
            wu=t(block.wu.weight.detach()[f0:f1]),
            wd=t(block.wd.weight.detach()[:, f0:f1]),
            heads=(h0, h1), ff=(f0, f1))
        if (dtype == torch.bfloat16 and sw.wg.is_cuda and f1 > f0 and (f1 - f0) % FF_UNIT == 0):
            from . import _torch_ops

            sw.wgu = _torch_ops.interleave_gate_up(sw.wg, sw.wu)
        return sw


def _device_ops():
    from . import ops

    return ops


class _Marks:
    """CUDA events recorded at the block's phase boundaries (for the bench's breakdown)."""

    def __init__(self, record: Optional[list]):
        self.record = record

    def __call__(self, name: str) -> None:
        if self.record is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.record.append((name, ev))


class sm_budget:
    """Context manager: the persistent GEMM and attention kernels launched from this host
    thread fill at most `sms` SMs (nkl_set_sm_budget; 0 = all), leaving the rest to kernels
    that run beside them, such as NCCL's."""

    def __init__(self, sms: int):
        self.sms = sms
        self.prev = 0

    def __enter__(self):
        from . import _native as N

        prev = ctypes.c_int(0)
        N.call("nkl_set_sm_budget", self.sms, ctypes.byref(prev))
        self.prev = prev.value
        return self

    def __exit__(self, *exc):
        from . import _native as N

        N.call("nkl_set_sm_budget", self.prev, None)


def decoder_block_overlapped(block, x: torch.Tensor, weights: Optional[ShardedBlockWeights] = None,
                             group=None, comm_sms: int = 0) -> torch.Tensor:
    """decoder_block for x [B, S, d] bf16 on CUDA with the collectives overlapped with the
    GEMMs: the batch elements go through the block one after another, each one's row
    all-gathers and fp32 reduce-scatters issued asynchronously (NCCL's stream) while the
    next element's projections and attention run. Rows are sharded per batch element
    (rank r holds rows shard_range(S, world, r) of every element, S % world == 0); every
    kernel, rounding point and fp32 reduction is that of decoder_block, row for row.
    With comm_sms > 0 the GEMM and attention grids leave that many SMs free (sm_budget)
    for NCCL's kernels; the result then equals decoder_block run under the same budget
    (the budget changes the attention's split-KV plan, and with it the rounding of split
    query tiles). On two B200s at B=4, S=4096, d=4096 that made the block slower (4.29 ms
    with all SMs, 4.42 ms with 16 left free, 4.50 ms with 32), so the default keeps every
    SM. Falls back to decoder_block when the shape does not allow it, and with four or more
    ranks."""
    world, rank = _world(group)
    B = x.shape[0] if x.dim() == 3 else 1
    cfg = block.cfg
    # With four or more ranks the per-element collectives are latency-bound and the serial
    # block is faster (eight B200s at B=4, S=4096, d=4096: 2.44 ms serial against 2.87 ms
    # overlapped; two: 5.06 ms serial against 4.29 ms overlapped).
    if (world == 1 or world >= 4 or x.dim() != 3 or B < 2 or x.shape[1] % world or not x.is_cuda
            or x.dtype != torch.bfloat16 or cfg.head_dim not in (64, 128)):
        return decoder_block(block, x, weights=weights, group=group)
    w = weights or shard_block(block, world, rank, x.dtype, x.device)
    sms = torch.cuda.get_device_properties(x.device).multi_processor_count
    with sm_budget(max(1, sms - comm_sms) if comm_sms > 0 else 0):
        return _overlapped(block, x, w, group, world, rank)


def _overlapped(block, x: torch.Tensor, w: ShardedBlockWeights, group, world: int, rank: int) -> torch.Tensor:
    cfg = block.cfg
    B, S, d = x.shape
    hd = cfg.head_dim
    nh = w.heads[1] - w.heads[0]
    s0, s1 = shard_range(S, world, rank)
    bf, f32 = torch.bfloat16, torch.float32
    dev = x.device
    x_loc = [x[b, s0:s1].contiguous() for b in range(B)]

    def ag(local):  # all-gather of one element's row shards, asynchronously
        full = torch.empty((S, d), dtype=local.dtype, device=dev)
        return full, dist.all_gather_into_tensor(full, local, group=group, async_op=True)

    def rs(part):  # fp32 reduce-scatter of one element's partial products, asynchronously
        out = torch.empty((s1 - s0, d), dtype=f32, device=dev)
        return out, dist.reduce_scatter_tensor(out, part, op=dist.ReduceOp.SUM, group=group, async_op=True)

    # attention half
    gathered = [ag(ops_rmsnorm(xl, w.norm1, cfg.eps)) for xl in x_loc]
    reduced = []
    for full, work in gathered:
        work.wait()  # the compute stream waits for the collective, the host does not
        if nh > 0:
            qkv = torch.ops.nkilab.matmul(full, w.wqkv, False).view(S, 3, nh, hd)
            a = torch.empty(S, nh, hd, dtype=bf, device=dev)
            q, k, v = (qkv[:, i].transpose(0, 1) for i in range(3))
            torch.ops.nkilab.attention_strided_(q, k, v, a.transpose(0, 1), 1.0 / math.sqrt(hd))
            part = torch.ops.nkilab.matmul_f32out(a.view(S, nh * hd), w.wo)
        else:
            part = torch.zeros((S, d), dtype=f32, device=dev)
        reduced.append(rs(part))
    # MLP half
    x1, gathered = [], []
    for xl, (attn_out, work) in zip(x_loc, reduced):
        work.wait()
        xb, hb = torch.ops.nkilab.add_rmsnorm(xl, attn_out.to(bf), w.norm2, cfg.eps)
        x1.append(xb)
        gathered.append(ag(hb))
    reduced = []
    for full, work in gathered:
        work.wait()
        if w.ff[1] > w.ff[0]:
            if w.wgu is not None:
                act = torch.ops.nkilab.matmul_swiglu(full, w.wgu)
            else:
                act = torch.ops.nkilab.swiglu(torch.ops.nkilab.matmul(full, w.wg, False),
                                              torch.ops.nkilab.matmul(full, w.wu, False))
            part = torch.ops.nkilab.matmul_f32out(act, w.wd)
        else:
            part = torch.zeros((S, d), dtype=f32, device=dev)
        reduced.append(rs(part))
    out = torch.empty((B, S, d), dtype=bf, device=dev)
    works = []
    for b, (xb, (mlp_out, work)) in enumerate(zip(x1, reduced)):
        work.wait()
        yb = (xb.float() + mlp_out.to(bf).float()).to(bf)
        works.append(dist.all_gather_into_tensor(out[b], yb, group=group, async_op=True))
    for work in works:
        work.wait()
    return out


def ops_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    return torch.ops.nkilab.rmsnorm(x, weight, eps)


def decoder_block(block, x: torch.Tensor, weights: Optional[ShardedBlockWeights] = None,
                  variant: str = "flash_pipelined", group=None, ops_module=None,
                  marks: Optional[list] = None) -> torch.Tensor:
    """Tensor-parallel DecoderBlock forward (nkilab/model.py:70-89, sharded).

    x: [S, d] or [B, S, d], the same full input on every rank (only this rank's row block
    of the flattened [B * S, d] rows is read). Returns the full output on every rank.

    Heads and FFN columns are split over the ranks, rows (sequence parallel) for the norms
    and residual adds. Per block: RMSNorm of the local rows -> all-gather -> QKV and causal
    attention of the local heads (per batch element) -> Wo partial in fp32 ->
    reduce-scatter (fp32 sum over ranks, one rounding to x's dtype: the rounding point of
    the single-GPU Wo product) -> residual add + RMSNorm of the local rows -> all-gather ->
    gate/up + SwiGLU of the local FFN columns -> Wd partial in fp32 -> reduce-scatter ->
    residual add -> all-gather of the block output. On CUDA bf16 the block uses the same
    fused kernels as the one-GPU path (strided attention over the QKV projection, fused
    residual add + RMSNorm, gate/up GEMM with SwiGLU in its epilogue) and fp32-output GEMMs
    for the partials. `marks`, if a list, receives (name, CUDA event) pairs at the phase
    boundaries."""
    world, rank = _world(group)
    dev_ops = ops_module is None
    if ops_module is None:
        from . import ops as ops_module
    mark = _Marks(marks)
    cfg = block.cfg
    lead = x.shape[:-1]
    S, d = x.shape[-2], x.shape[-1]
    B = x[..., 0, 0].numel() if x.dim() == 3 else 1
    R = B * S
    hd = cfg.head_dim
    dt = x.dtype
    w = weights or shard_block(block, world, rank, dt, x.device)
    nh = w.heads[1] - w.heads[0]
    r0, r1 = shard_range(R, world, rank)
    x_loc = x.reshape(R, d)[r0:r1].contiguous()
    fused = dev_ops and x.is_cuda and dt == torch.bfloat16

    def partial_f32(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        if fused:
            return torch.ops.nkilab.matmul_f32out(a.contiguous(), b)
        f32 = getattr(ops_module, "matmul_f32", None)
        return f32(a, b) if f32 is not None else ops_module.matmul(a, b).float()

    # ---- attention half
    mark("start")
    h_loc = ops_module.rmsnorm(x_loc, w.norm1, cfg.eps)
    mark("norm1")
    h = all_gather_dim0(h_loc, R, group)
    mark("all_gather_1")
    if nh > 0:
        qkv = ops_module.matmul(h, w.wqkv)  # [R, 3 * nh * hd]
        if fused and variant != "naive" and hd in (64, 128):
            a = torch.empty(R, nh * hd, dtype=dt, device=x.device)
            qkv3 = qkv.view(B, S, 3, nh, hd)
            a3 = a.view(B, S, nh, hd)
            for b in range(B):  # local heads read straight out of the projection, output in the Wo layout
                q, k, v = (qkv3[b, :, i].transpose(0, 1) for i in range(3))
                torch.ops.nkilab.attention_strided_(q, k, v, a3[b].transpose(0, 1), 1.0 / math.sqrt(hd))
        else:
            q, k, v = (qkv[:, i * nh * hd:(i + 1) * nh * hd].reshape(B, S, nh, hd).permute(0, 2, 1, 3)
                       .reshape(B * nh, S, hd).contiguous() for i in range(3))
            a = ops_module.attention(q, k, v, variant=variant)
            a = a.view(B, nh, S, hd).permute(0, 2, 1, 3).reshape(R, nh * hd).contiguous()
        part = partial_f32(a, w.wo)
    else:
        part = torch.zeros((R, d), dtype=torch.float32, device=x.device)
    mark("attention")
    attn_out = reduce_scatter_dim0(part, group).to(dt)  # fp32 sum over ranks, one rounding
    mark("reduce_scatter_1")
    if fused:
        x_loc, h_loc = torch.ops.nkilab.add_rmsnorm(x_loc, attn_out.contiguous(), w.norm2, cfg.eps)
    else:
        x_loc = (x_loc.float() + attn_out.float()).to(dt)
        h_loc = ops_module.rmsnorm(x_loc, w.norm2, cfg.eps)
    mark("norm2")
    # ---- MLP half
    h = all_gather_dim0(h_loc, R, group)
    mark("all_gather_2")
    if w.ff[1] > w.ff[0]:
        if fused and w.wgu is not None:
            act = torch.ops.nkilab.matmul_swiglu(h, w.wgu)
        else:
            act = ops_module.swiglu(ops_module.matmul(h, w.wg), ops_module.matmul(h, w.wu))
        part = partial_f32(act, w.wd)
    else:
        part = torch.zeros((R, d), dtype=torch.float32, device=x.device)
    mark("mlp")
    mlp_out = reduce_scatter_dim0(part, group).to(dt)
    mark("reduce_scatter_2")
    y_loc = (x_loc.float() + mlp_out.float()).to(dt)
    out = all_gather_dim0(y_loc, R, group)
    mark("all_gather_3")
    return out.view(*lead, d)

"""Multi-rank logic of nkilab.parallel on CPU: world_size-2 gloo process groups.

The per-shard compute is the CPU oracle (injected through the modules' `compute` /
`ops_module` hooks, test-only), so these tests check the sharding, padding, gather and
reduce-scatter logic and its results, not the kernels. A failure test makes one rank
leave before a collective and checks that the other rank gets an error from the
process-group timeout instead of hanging."""
from __future__ import annotations

import datetime
import os
import socket
import types

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import nki_oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _oracle_ops():
    def attention(q, k, v, variant="flash_pipelined"):
        return (O.attention_naive if variant == "naive" else O.attention_flash)(q, k, v)

    return types.SimpleNamespace(rmsnorm=O.rmsnorm, matmul=O.matmul, swiglu=O.swiglu, attention=attention,
                                 matmul_f32=lambda a, b: a.float() @ b.float())


def _row_compute(op, *args, **kw):
    if op == "rmsnorm":
        return O.rmsnorm(*args, **kw)
    if op == "softmax":
        return O.softmax_fused(*args)
    return O.swiglu(*args)


def _worker_collectives(rank, world, port):
    from nkilab import parallel as P

    _init(rank, world, port)
    try:
        # uneven all-gather: 7 rows over `world` ranks
        r0, r1 = P.shard_range(7, world, rank)
        local = torch.arange(r0, r1, dtype=torch.float32).view(-1, 1).repeat(1, 3)
        full = P.all_gather_dim0(local, 7)
        assert torch.equal(full[:, 0], torch.arange(7, dtype=torch.float32))
        # reduce-scatter: every rank contributes (rank + 1) * base
        base = torch.arange(5 * 2, dtype=torch.float32).view(5, 2)
        part = P.reduce_scatter_dim0(base * (rank + 1))
        s0, s1 = P.shard_range(5, world, rank)
        assert torch.allclose(part, base[s0:s1] * sum(r + 1 for r in range(world)))
        # row kernels, sharded by rows
        g = torch.Generator().manual_seed(3)
        x = torch.randn(9, 64, generator=g)
        u = torch.randn(9, 64, generator=g)
        w = torch.rand(64, generator=g) + 0.5
        assert torch.equal(P.row_op("rmsnorm", x, w, compute=_row_compute, eps=1e-6), O.rmsnorm(x, w, 1e-6))
        assert torch.equal(P.row_op("softmax", x, compute=_row_compute), O.softmax_fused(x))
        assert torch.equal(P.row_op("swiglu", x, u, compute=_row_compute), O.swiglu(x, u))
        # attention, sharded by heads (3 heads over 2 ranks: uneven)
        q, k, v = (torch.randn(3, 200, 32, generator=g) for _ in range(3))
        ops = _oracle_ops()
        out = P.attention(q, k, v, compute=lambda a, b, c, var: ops.attention(a, b, c, var))
        assert torch.equal(out, O.attention_flash(q, k, v))
        # GEMM, columns of b sharded in 128-column units (300 columns: uneven, last unit partial)
        a = torch.randn(17, 40, generator=g)
        b = torch.randn(40, 300, generator=g)
        c = P.matmul(a, b, compute=O.matmul)
        assert c.shape == (17, 300)
        assert torch.equal(c, O.matmul(a, b))
    finally:
        dist.destroy_process_group()


def _worker_block(rank, world, port):
    from nkilab import parallel as P
    from nkilab.model import BlockConfig, DecoderBlock

    _init(rank, world, port)
    try:
        torch.manual_seed(0)
        block = DecoderBlock(BlockConfig(d_model=256, n_heads=4, d_ff=1000)).eval()
        x = torch.randn(130, 256, generator=torch.Generator().manual_seed(1))
        with torch.no_grad():
            ref = block(x)
        out = P.decoder_block(block, x, ops_module=_oracle_ops())
        assert out.shape == x.shape
        assert float((out - ref).abs().max()) < 1e-5, float((out - ref).abs().max())
        # batched input [B, S, d]: rows of all batch elements are sharded together, attention
        # stays within each element; the phase marks come back in order
        xb = torch.randn(3, 40, 256, generator=torch.Generator().manual_seed(2))
        with torch.no_grad():
            refb = torch.stack([block(xb[i]) for i in range(3)])
        outb = P.decoder_block(block, xb, ops_module=_oracle_ops())
        assert outb.shape == xb.shape
        assert float((outb - refb).abs().max()) < 1e-5, float((outb - refb).abs().max())
        # FFN columns in whole 128-column units: d_ff=1000 -> 8 units, 4 per rank
        f0, f1 = P.ff_range(1000, world, rank)
        assert (f0, f1) == ((0, 512) if rank == 0 else (512, 1000))
    finally:
        dist.destroy_process_group()


def _worker_rank_leaves(rank, world, port, q):
    _init(rank, world, port, timeout_s=3)
    if rank == 1:
        return  # leaves between steps, never joins the collective
    t = torch.ones(2)
    try:
        dist.all_reduce(t)
        q.put("completed")
    except Exception as e:  # the surviving rank must see an error, not hang
        q.put(f"error: {type(e).__name__}")


def test_shard_range_covers_evenly():
    from nkilab import parallel as P

    for n in range(0, 40):
        for world in range(1, 9):
            parts = [P.shard_range(n, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            sizes = [e - s for s, e in parts]
            assert max(sizes) - min(sizes) <= 1


def test_collectives_rows_and_heads_world2():
    mp.spawn(_worker_collectives, args=(2, _free_port()), nprocs=2, join=True)


def test_tensor_parallel_decoder_block_world2():
    mp.spawn(_worker_block, args=(2, _free_port()), nprocs=2, join=True)


def test_rank_that_leaves_is_detected_by_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_rank_leaves, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode is not None for p in procs), "a rank hung"
    result = q.get(timeout=5)
    assert result.startswith("error"), result

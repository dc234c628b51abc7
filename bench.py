"""Benchmark of the nkilab B200 kernel set (prints ONE JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (BASELINE.json metric): causal flash attention, 8 heads x 2048 x 128, bf16,
one forward per step. On one GPU the whole problem runs on it; on N GPUs (torchrun, one
process per GPU) the same fixed problem is sharded by heads (strong scaling): rank r
computes heads shard_range(8, N, r), then one NCCL all-gather assembles the full output
on every rank, both inside the timed region. Also on the same line: the row kernels at
[4096, 2048] bf16 (HBM GB/s), the GEMM at 1024^3 and 8192^3 bf16, and the decoder block
of BASELINE's configs[4] (tensor-parallel over the N GPUs), each against the measured
roofline; at N > 1 also N independent replicas of the headline (weak scaling) and the
sharded results' parity against one GPU.

value      K steps through torch.ops.nkilab.attention (+ the all-gather at N > 1),
           captured in one CUDA graph, inputs resident in HBM, rotating through a
           256 MiB pool of input sets so no step finds its inputs in the 126 MB L2; the
           graph replayed 7 times, each replay timed with CUDA events on the launching
           stream, barrier + synchronize on both sides; the median replay, max over
           ranks (step_us_spread: median / min / max per step on rank 0). value =
           8.59e9 FLOP / that time (the whole job). The row kernels are timed the same
           way (frac at the median, frac_min / frac_max at the slowest / fastest replay).
e2e        the same metric through the public API with pinned host tensors
           (nkilab.ops.attention on one GPU, nkilab.parallel.attention on N): host->device
           copy of q, k, v and device->host copy of the output inside every timed step.
reference  --impl reference times the reference algorithm on the host cores: the
           CPU port of the NKI kernels (oracle/nki_oracle.py), since the reference's
           own CPU path (the NKI simulator) cannot be installed in this image.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nki-kernel-lab_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

H, S, D = 8, 2048, 128
ATTN_FLOP = 2.0 * H * S * S * D  # causal half of 4*H*S^2*d
ROWS, COLS = 4096, 2048
METRIC = "causal-attn TFLOPS (8×2048×128 bf16) + row-kernel HBM GB/s, % roofline"
L2_BYTES = 126 * 1024 * 1024
POOL_BYTES = 256 * 1024 * 1024


def peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def ncu_traffic(kernel_file: str, key: str = ""):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/<kernel_file>: the
    line 'traffic_bytes_per_launch[ key]: N'."""
    try:
        with open(os.path.join(ROOT, "profiles", kernel_file)) as f:
            pat = r"traffic_bytes_per_launch" + (r"\s+" + re.escape(key) if key else "") + r":\s*([0-9.eE+]+)"
            m = re.search(pat, f.read())
        return float(m.group(1)) if m else None
    except OSError:
        return None


# --------------------------------------------------------------------------- clocks

class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = os.path.join("/tmp", f"nkl_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        loaded = [float(r[1]) for r in rows if r[3].replace(".", "").isdigit() and float(r[3]) > 250.0] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------- timing helpers

REPLAYS = 7  # timed replays of every captured graph; the median is reported


def timed_graph_runs(fn_step, n_steps: int, stream: torch.cuda.Stream, replays: int = REPLAYS) -> list:
    """Capture n_steps calls of fn_step(i) in one CUDA graph; return the elapsed ms of each
    of `replays` replays, measured with CUDA events on `stream`. One untimed replay first
    uploads the graph to the device (a one-time cost of the first launch, not of the
    steps)."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            for i in range(n_steps):
                fn_step(i)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize()
    out = []
    for _ in range(replays):
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            t0.record(stream)
            g.replay()
            t1.record(stream)
        torch.cuda.synchronize()
        out.append(t0.elapsed_time(t1))
    del g
    return out


def timed_graph(fn_step, n_steps: int, stream: torch.cuda.Stream) -> float:
    """Median over REPLAYS timed replays of the n_steps graph (ms for all n_steps)."""
    return statistics.median(timed_graph_runs(fn_step, n_steps, stream))


def spread(runs: list, n_steps: int, scale: float = 1e3) -> dict:
    """Median, min and max per step of a list of per-replay times (ms), in us by default."""
    per = sorted(r / n_steps * scale for r in runs)
    return {"median": round(statistics.median(per), 3), "min": round(per[0], 3), "max": round(per[-1], 3),
            "replays": len(per)}


def warm(fn_step, n: int, stream):
    with torch.cuda.stream(stream):
        for i in range(n):
            fn_step(i)
    torch.cuda.synchronize()


# --------------------------------------------------------------------------- our arm

def bench_attention(steps: int, warmup: int, dev, stream, dist_ctx) -> dict:
    per_set = 4 * H * S * D * 2
    nset = max(2, math.ceil(POOL_BYTES / per_set))
    g = torch.Generator(device=dev).manual_seed(1234 + dist_ctx["rank"])
    pool = [tuple(torch.randn(H, S, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
            for _ in range(nset)]
    scale = 1.0 / math.sqrt(D)

    keep = []  # every step's output stays alive, so each step writes fresh memory (not an L2-resident buffer)

    def step(i):
        q, k, v = pool[i % nset]
        keep.append(torch.ops.nkilab.attention(q, k, v, scale, False))
        if len(keep) > 2 * steps + 8:
            keep.pop(0)

    warm(step, warmup, stream)
    # clock soak: same load, untimed, so the 200 ms clock samples see the kernel running
    t_end = time.time() + 1.5
    while time.time() < t_end:
        warm(step, 200, stream)
    dist_ctx["barrier"]()
    torch.cuda.synchronize()
    runs = timed_graph_runs(step, steps, stream)
    torch.cuda.synchronize()
    dist_ctx["barrier"]()
    ms = dist_ctx["max"](statistics.median(runs))
    # One op = the attention kernel, plus the split-KV combine kernel when the plan for
    # this shape splits key ranges (it does whenever a workspace is needed).
    from nkilab import _native
    split = _native.lib.nkl_attention_workspace_size(H, S, D, _native.BFLOAT16) > 0
    return {"ms_total": ms, "ms_per_step": ms / steps, "pool_sets": nset, "pool_mib": nset * per_set / 2**20,
            "launches_per_step": 2 if split else 1}


def bench_attention_sharded(steps: int, warmup: int, dev, stream, ctx, gather: str = "nvlink") -> dict:
    """Head-sharded attention on the fixed 8x2048x128 problem (strong scaling): rank r
    computes heads shard_range(8, N, r) and the full [8, 2048, 128] output is assembled on
    every rank inside the timed CUDA graph -- by the attention kernels themselves over
    NVLink (gather="nvlink", parallel.PeerAttention: output tiles stored into every rank's
    buffer, then a flag exchange) or by an NCCL all-gather after them (gather="nccl"). The
    same steps without any gather are timed separately to split out the collective."""
    from nkilab import _native
    from nkilab import parallel as P

    world, rank = ctx["world"], ctx["rank"]
    peer = P.PeerAttention(H, S, D, device=dev) if (gather == "nvlink" and world > 1) else None
    h0, h1 = P.shard_range(H, world, rank)
    hl = h1 - h0
    per_set = 3 * hl * S * D * 2
    nset = max(2, math.ceil(POOL_BYTES / per_set))
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    pool = [tuple(torch.randn(hl, S, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
            for _ in range(nset)]
    scale = 1.0 / math.sqrt(D)
    keep = []

    def step(i, gather=True):
        q, k, v = pool[i % nset]
        if gather and peer is not None:
            keep.append(peer(q, k, v))
        else:
            local = torch.ops.nkilab.attention(q, k, v, scale, False)
            keep.append(P.all_gather_dim0(local, H) if gather else local)
        if len(keep) > 2 * steps + 8:
            keep.pop(0)

    warm(step, warmup, stream)
    t_end = time.time() + 1.0
    while time.time() < t_end:
        warm(step, 100, stream)
    ctx["barrier"]()
    torch.cuda.synchronize()
    runs = timed_graph_runs(step, steps, stream)
    ms = ctx["max"](statistics.median(runs))
    keep.clear()
    ctx["barrier"]()
    ms_compute = ctx["max"](timed_graph(lambda i: step(i, gather=False), steps, stream))
    keep.clear()
    if peer is not None:
        torch.cuda.synchronize()
        _native.check_device(stream.cuda_stream)  # the flag exchange never timed out
        peer.close()
    split = _native.lib.nkl_attention_workspace_size(hl, S, D, _native.BFLOAT16) > 0
    return {"ms_total": ms, "ms_per_step": ms / steps, "pool_sets": nset, "pool_mib": nset * per_set / 2**20,
            "gather": gather if world > 1 else "none",
            "launches_per_step": (2 if split else 1) + (1 if peer is not None else 0), "heads_per_rank": hl,
            "us_per_step_rank0": spread(runs, steps),
            "attention_us": round(ms_compute / steps * 1e3, 3),
            "all_gather_us": round((ms - ms_compute) / steps * 1e3, 3) if world > 1 else 0.0}


def sharded_parity(dev, ctx) -> dict:
    """Before timing: the head-sharded attention (all-gathered on every rank) against
    attention of all heads on one GPU (rank 0), on the same inputs."""
    from nkilab import ops
    from nkilab import parallel as P

    g = torch.Generator(device=dev).manual_seed(77)
    q, k, v = (torch.randn(H, S, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
    got = P.attention(q, k, v)
    peer = P.PeerAttention(H, S, D, device=dev)
    h0, h1 = P.shard_range(H, ctx["world"], ctx["rank"])
    got_p2p = peer(*(t[h0:h1].contiguous() for t in (q, k, v))).clone()
    torch.cuda.synchronize()
    peer.close()
    out = {}
    if ctx["rank"] == 0:
        ref = ops.attention(q, k, v)
        out["attn_rel_err"] = _rel(got, ref)
        out["attn_nvlink_gather_rel_err"] = _rel(got_p2p, ref)
        out["nvlink_gather_equals_nccl_gather"] = bool(torch.equal(got_p2p, got))
    return out


def _rel(a, b) -> float:
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-12))


def bench_rows(steps: int, warmup: int, dev, stream, pk) -> dict:
    """Row kernels through the C ABI with rotating input AND output buffers (a pool larger
    than 2x L2), so neither the reads nor the writes of a step hit lines an earlier step
    left in L2."""
    from nkilab import _native as N

    out = {}
    g = torch.Generator(device=dev).manual_seed(7)
    x_bytes = ROWS * COLS * 2
    specs = {
        "rmsnorm": (2, 2 * x_bytes + COLS * 2),
        "softmax": (1, 2 * x_bytes),
        "swiglu": (2, 3 * x_bytes),
    }
    st = stream.cuda_stream
    for name, (n_in, alg_bytes) in specs.items():
        nset = max(2, math.ceil(POOL_BYTES / (alg_bytes)))
        sets = [[torch.randn(ROWS, COLS, device=dev, generator=g).to(torch.bfloat16) for _ in range(n_in)]
                + [torch.empty(ROWS, COLS, device=dev, dtype=torch.bfloat16)] for _ in range(nset)]
        gamma = (1 + 0.1 * torch.randn(COLS, device=dev, generator=g)).to(torch.bfloat16)

        def step(i, name=name, sets=sets, gamma=gamma):
            t = sets[i % len(sets)]
            if name == "rmsnorm":
                N.call("nkl_rmsnorm", t[0].data_ptr(), gamma.data_ptr(), t[-1].data_ptr(), ROWS, COLS, 1e-6,
                       N.BFLOAT16, st)
            elif name == "softmax":
                N.call("nkl_softmax", t[0].data_ptr(), t[-1].data_ptr(), ROWS, COLS, N.BFLOAT16, st)
            else:
                N.call("nkl_swiglu", t[0].data_ptr(), t[1].data_ptr(), t[-1].data_ptr(), ROWS, COLS, N.BFLOAT16, st)

        warm(step, warmup, stream)
        runs = timed_graph_runs(step, steps, stream)
        ms = statistics.median(runs) / steps
        gbs = alg_bytes / (ms * 1e-3) / 1e9
        sp = spread(runs, steps)
        out[name] = {"us": round(ms * 1e3, 3), "gbs": round(gbs, 1), "frac": round(gbs / pk["hbm_gbs"], 4),
                     "traffic_bytes_per_launch": ncu_traffic("rows_bf16_4096x2048.md", name),
                     "frac_min": round(alg_bytes / (sp["max"] * 1e-6) / 1e9 / pk["hbm_gbs"], 4),
                     "frac_max": round(alg_bytes / (sp["min"] * 1e-6) / 1e9 / pk["hbm_gbs"], 4),
                     "us_spread": sp, "bytes_per_launch": alg_bytes, "pool_mib": round(nset * alg_bytes / 2**20),
                     "outputs": "rotating with the inputs"}
        del sets
    return out


def bench_gemm(dev, stream, pk) -> dict:
    out = {}
    for n, steps in ((1024, 200), (8192, 10)):
        g = torch.Generator(device=dev).manual_seed(n)
        per = 3 * n * n * 2
        nset = max(1, math.ceil(POOL_BYTES / per)) if n <= 4096 else 1
        sets = [((torch.rand(n, n, device=dev, generator=g) * 2 - 1).to(torch.bfloat16),
                 (torch.rand(n, n, device=dev, generator=g) * 2 - 1).to(torch.bfloat16)) for _ in range(nset)]

        def step(i, sets=sets):
            a, b = sets[i % len(sets)]
            torch.ops.nkilab.matmul(a, b, False)

        def cublas(i, sets=sets):
            a, b = sets[i % len(sets)]
            torch.matmul(a, b)

        warm(step, 3, stream)
        ms = timed_graph(step, steps, stream) / steps
        warm(cublas, 3, stream)
        ms_cublas = timed_graph(cublas, steps, stream) / steps  # the library GEMM, same inputs and harness
        tf = 2.0 * n ** 3 / (ms * 1e-3) / 1e12
        out[f"{n}^3"] = {"us": round(ms * 1e3, 2), "tflops": round(tf, 1), "frac": round(tf / pk["bf16_tflops"], 4),
                         "cublas_us_same_run": round(ms_cublas * 1e3, 2),
                         "traffic_bytes_per_launch": ncu_traffic("gemm_bf16_1024_8192.md", str(n))}
        del sets
    return out


def make_block(dev, ctx):
    """BASELINE configs[4]'s block with bf16-representable random weights ~ N(0, 0.02) and
    norm gains ~ U(0.5, 1.5), made on rank 0 and broadcast so every rank holds the same."""
    from nkilab.model import BlockConfig, DecoderBlock

    cfg = BlockConfig(d_model=4096, n_heads=32, d_ff=11008)
    with torch.device("meta"):
        block = DecoderBlock(cfg)
    block = block.to_empty(device=dev)
    g = torch.Generator(device=dev).manual_seed(0)
    with torch.no_grad():
        for p in block.parameters():
            p.normal_(0.0, 0.02, generator=g)
        block.norm1.weight.uniform_(0.5, 1.5, generator=g)
        block.norm2.weight.uniform_(0.5, 1.5, generator=g)
        if ctx["world"] > 1:
            import torch.distributed as dist

            for p in block.parameters():
                dist.broadcast(p.data, 0)
    return block


def bench_block(dev, stream, pk, ctx) -> dict:
    """The decoder block of BASELINE configs[4] (B=4, S=4096, d=4096, 32x128 heads,
    ff=11008, bf16). One GPU: nkilab.model.nki_forward. N GPUs: nkilab.parallel's
    tensor-parallel block (heads and FFN columns sharded, rows sequence-parallel, fp32
    partials reduce-scattered), timed per step as the max over ranks, with the time of
    each collective (CUDA events at the phase boundaries, rank 0) split out. Before
    timing, rank 0 compares the sharded output with nki_forward on one GPU."""
    from nkilab import parallel as P
    from nkilab.model import nki_forward

    world, rank = ctx["world"], ctx["rank"]
    block = make_block(dev, ctx)
    B, Sb, d, f = 4, 4096, 4096, 11008
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(B, Sb, d, device=dev, generator=g).to(torch.bfloat16)
    flop = 2.0 * B * Sb * d * (3 * d + d + 2 * f) + 2.0 * B * Sb * f * d + 2.0 * B * 32 * Sb * Sb * 128
    out = {"config": "B=4 S=4096 d=4096 H=32x128 ff=11008 bf16", "flop": flop}
    if world == 1:
        fwd = lambda: nki_forward(block, x)  # noqa: E731
        out["parallelism"] = "single"
    else:
        w = P.shard_block(block, world, rank, torch.bfloat16, dev)
        serial = lambda marks=None: P.decoder_block(block, x, weights=w, marks=marks)  # noqa: E731
        fwd = lambda: P.decoder_block_overlapped(block, x, weights=w)  # noqa: E731
        out["parallelism"] = (f"tp{world} heads x ffn columns, sequence-parallel rows, fp32 reduce-scatter; "
                              + ("collectives of each batch element overlapped with the next one's GEMMs"
                                 if world < 4 else "serial (parallel.decoder_block_overlapped falls back to it "
                                                   "from four ranks on)"))
        with torch.cuda.stream(stream):
            y = fwd()
            torch.cuda.synchronize()
            if rank == 0:
                ref = nki_forward(block, x)
                diff = (y.float() - ref.float()).abs()
                out["parity_vs_one_gpu"] = {"rel_err": _rel(y, ref), "mean_abs_err": float(diff.mean()),
                                            "elements_differing": float((diff > 0).float().mean()),
                                            "note": "one-GPU block vs the CPU oracle differs by the same "
                                                    "one-ulp output flips (tests/test_model_gpu.py)"}
                del ref
            del y
        block.__dict__.pop("_nkl_weight_cache", None)
    with torch.cuda.stream(stream):
        for _ in range(2):
            fwd()
        torch.cuda.synchronize()
        ctx["barrier"]()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        steps = 10  # ~50 ms per variant; 3 steps left the variants' order to noise at two GPUs
        t0.record(stream)
        for _ in range(steps):
            fwd()
        t1.record(stream)
        torch.cuda.synchronize()
        ms = ctx["max"](t0.elapsed_time(t1) / steps)
        if world > 1:  # SMs left to NCCL while the overlapped block's GEMMs run
            by_sms = {}
            for c in ((16, 32) if world < 4 else ()):
                ctx["barrier"]()
                P.decoder_block_overlapped(block, x, weights=w, comm_sms=c)
                torch.cuda.synchronize()
                ctx["barrier"]()
                t0.record(stream)
                for _ in range(steps):
                    P.decoder_block_overlapped(block, x, weights=w, comm_sms=c)
                t1.record(stream)
                torch.cuda.synchronize()
                by_sms[c] = round(ctx["max"](t0.elapsed_time(t1) / steps), 3)
            by_sms[0] = round(ms, 3)
            out["ms_by_comm_sms"] = {str(k): by_sms[k] for k in sorted(by_sms)}
        if world > 1:  # the same block without the overlap, with events at the phase boundaries
            ctx["barrier"]()
            for _ in range(2):
                serial()
            torch.cuda.synchronize()
            ctx["barrier"]()
            t0.record(stream)
            for _ in range(steps):
                serial()
            t1.record(stream)
            torch.cuda.synchronize()
            out["ms_without_overlap"] = round(ctx["max"](t0.elapsed_time(t1) / steps), 3)
            ctx["barrier"]()
            marks = []
            serial(marks)
            torch.cuda.synchronize()
            names = [n for n, _ in marks]
            spans = {names[i]: marks[i - 1][1].elapsed_time(marks[i][1]) for i in range(1, len(marks))}
            coll = {k: round(v * 1e3, 1) for k, v in spans.items() if k.startswith(("all_gather", "reduce_scatter"))}
            out["breakdown_us_rank0"] = {k: round(v * 1e3, 1) for k, v in spans.items()}
            out["collective_us_rank0"] = round(sum(coll.values()), 1)
            out["limiter"] = max(spans, key=spans.get)
    tf = flop / (ms * 1e-3) / 1e12
    out.update({"ms": round(ms, 3), "tflops": round(tf, 1),
                "frac": round(tf / (world * pk["bf16_tflops_sustained"]), 4)})
    del block
    return out


def bench_ladder(dev, stream, pk) -> dict:
    """The reference's variant ladder (README.md:17-23, bench/run_bench.py:108-138) as
    measured B200 rungs, each a distinct kernel or launch mode, graph-timed like the
    headline (median of 7 replays, rotating inputs larger than L2):
      attention 8x2048x128: naive (scores and probabilities through HBM) -> flash, one
      query tile per CTA, no split (flash / flash_kv_resident) -> the same kernel with
      causal key ranges split over all SMs (flash_balanced; the default) -> two query
      tiles per CTA interleaved (flash_pipelined's ILP = 2) -> one query tile, two softmax
      groups on alternate key tiles
      softmax [4096, 2048]: unfused (3 HBM passes) -> fused; GEMM 1024^3: naive -> blocked."""
    from nkilab import _native as N

    out = {}
    scale = 1.0 / math.sqrt(D)
    per = 4 * H * S * D * 2
    nset = max(2, math.ceil(POOL_BYTES / per))
    g = torch.Generator(device=dev).manual_seed(21)
    sets = [[torch.randn(H, S, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(4)] for _ in range(nset)]
    st = stream.cuda_stream
    att = {}
    for name, mode in (("flash_one_tile_unsplit", N.ATTN_ONE_TILE_UNSPLIT), ("flash_split_kv_default", N.ATTN_AUTO),
                       ("flash_two_tile", N.ATTN_TWO_TILE), ("flash_two_softmax_groups", N.ATTN_TWO_GROUPS)):
        nbytes = N.lib.nkl_attention_mode_workspace_size(H, S, D, N.BFLOAT16, mode)
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)

        def step(i, mode=mode, ws=ws, nbytes=nbytes):
            q, k, v, o = sets[i % nset]
            N.call("nkl_attention_mode", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), ws.data_ptr(), nbytes,
                   H, S, D, scale, N.BFLOAT16, mode, st)

        warm(step, 3, stream)
        us = statistics.median(timed_graph_runs(step, 20, stream)) / 20 * 1e3
        att[name] = {"us": round(us, 2), "tflops": round(ATTN_FLOP / (us * 1e-6) / 1e12, 1)}
    nb = N.lib.nkl_attention_naive_workspace_size(H, S, N.BFLOAT16)
    wsn = torch.empty(nb, dtype=torch.uint8, device=dev)

    def naive(i):
        q, k, v, o = sets[i % nset]
        N.call("nkl_attention_naive", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), wsn.data_ptr(), nb, H, S,
               D, scale, N.BFLOAT16, st)

    warm(naive, 2, stream)
    us = statistics.median(timed_graph_runs(naive, 3, stream, replays=3)) / 3 * 1e3
    att = {"naive": {"us": round(us, 1), "tflops": round(ATTN_FLOP / (us * 1e-6) / 1e12, 2)}, **att}
    del wsn, sets
    out["attention_8x2048x128"] = att
    x = [torch.randn(ROWS, COLS, device=dev, generator=g).to(torch.bfloat16) for _ in range(8)]
    y = torch.empty_like(x[0])
    wb = N.lib.nkl_softmax_unfused_workspace_size(ROWS, COLS)
    wsu = torch.empty(wb, dtype=torch.uint8, device=dev)
    sm = {}
    for name in ("unfused", "fused"):
        def step(i, name=name):
            t = x[i % len(x)]
            if name == "fused":
                N.call("nkl_softmax", t.data_ptr(), y.data_ptr(), ROWS, COLS, N.BFLOAT16, st)
            else:
                N.call("nkl_softmax_unfused", t.data_ptr(), y.data_ptr(), wsu.data_ptr(), wb, ROWS, COLS, N.BFLOAT16, st)

        warm(step, 3, stream)
        us = statistics.median(timed_graph_runs(step, 20, stream)) / 20 * 1e3
        sm[name] = {"us": round(us, 2), "gbs_algorithmic": round(2 * ROWS * COLS * 2 / (us * 1e-6) / 1e9, 1)}
    out["softmax_4096x2048"] = sm
    del x, wsu
    n = 1024
    mats = [[(torch.rand(n, n, device=dev, generator=g) * 2 - 1).to(torch.bfloat16) for _ in range(3)] for _ in range(16)]
    gm = {}
    for name in ("naive", "blocked"):
        def step(i, name=name):
            a, b, c = mats[i % len(mats)]
            N.call("nkl_matmul_naive" if name == "naive" else "nkl_matmul", a.data_ptr(), b.data_ptr(), c.data_ptr(), n, n,
                   n, N.BFLOAT16, st)

        warm(step, 3, stream)
        us = statistics.median(timed_graph_runs(step, 10, stream)) / 10 * 1e3
        gm[name] = {"us": round(us, 2), "tflops": round(2.0 * n ** 3 / (us * 1e-6) / 1e12, 1)}
    out["gemm_1024"] = gm
    return out


def bench_e2e(steps: int, warmup: int, dev, ctx) -> dict:
    """The headline through the public API with pinned host tensors: nkilab.ops.attention
    on one GPU, nkilab.parallel.attention on N (each rank copies its heads in, the
    gathered output comes back to every rank's host)."""
    from nkilab import ops
    from nkilab import parallel as P

    world, rank = ctx["world"], ctx["rank"]
    fn = ops.attention if world == 1 else P.attention
    g = torch.Generator().manual_seed(99)
    host = [torch.randn(H, S, D, generator=g).to(torch.bfloat16).pin_memory() for _ in range(3)]
    # Untimed warm-up of at least 50 calls (~25 ms): measured alone, the first ~30-40 host
    # round trips of a process run 1.5-1.7x slower than the steady state.
    for _ in range(max(50, warmup)):
        fn(*host)
    torch.cuda.synchronize()
    ctx["barrier"]()
    stream = torch.cuda.current_stream(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        out = fn(*host)  # H2D of q, k, v (this rank's heads); kernels (+ all-gather); D2H of out
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / steps
    assert out.shape == (H, S, D)
    h0, h1 = (0, H) if world == 1 else P.shard_range(H, world, rank)
    return {"value": round(ATTN_FLOP / (ms * 1e-3) / 1e12, 3), "unit": "TFLOPS", "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": 3 * (h1 - h0) * S * D * 2, "d2h_bytes_per_step": H * S * D * 2,
            "api": "nkilab.ops.attention" if world == 1 else "nkilab.parallel.attention",
            "bytes_scope": "per GPU" if world > 1 else "the one GPU"}


# --------------------------------------------------------------------------- CPU baselines

def cpu_attention_baseline(budget_s: float = 12.0) -> dict:
    """The reference algorithm on host cores: oracle port of flash_attention_pipelined
    (tile-level restatement, fp32 with bf16 P) on the full 8 x 2048 x 128 workload,
    repeated within a wall-clock budget; plus torch SDPA (the reference tests' own
    PyTorch reference) on the same inputs."""
    from oracle import nki_oracle as O

    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(H, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
    O.attention_flash(q[:1, :256], k[:1, :256], v[:1, :256])
    reps, t0 = 0, time.perf_counter()
    while True:
        O.attention_flash(q, k, v)
        reps += 1
        el = time.perf_counter() - t0
        if el > budget_s or reps >= 50:
            break
    port_tflops = ATTN_FLOP * reps / el / 1e12
    qf, kf, vf = q.float(), k.float(), v.float()
    torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, is_causal=True)
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < 3.0:
        torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, is_causal=True)
        n += 1
    sdpa_tflops = ATTN_FLOP * n / (time.perf_counter() - t0) / 1e12
    return {"value": round(port_tflops, 5), "unit": "TFLOPS", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{reps} full steps of oracle flash attention 8x2048x128 (bf16 in, fp32 math) in {el:.1f} s",
            "torch_sdpa_fp32_tflops": round(sdpa_tflops, 5), "host_cpus": os.cpu_count()}


def cpu_rows_baseline() -> dict:
    from oracle import nki_oracle as O

    g = torch.Generator().manual_seed(6)
    x = torch.randn(ROWS, COLS, generator=g).to(torch.bfloat16)
    u = torch.randn(ROWS, COLS, generator=g).to(torch.bfloat16)
    w = torch.ones(COLS).to(torch.bfloat16)
    out = {}
    for name, fn, nbytes in (("rmsnorm", lambda: O.rmsnorm(x, w), 2 * ROWS * COLS * 2 + COLS * 2),
                             ("softmax", lambda: O.softmax_fused(x), 2 * ROWS * COLS * 2),
                             ("swiglu", lambda: O.swiglu(x, u), 3 * ROWS * COLS * 2)):
        fn()
        t0, n = time.perf_counter(), 0
        while time.perf_counter() - t0 < 1.0:
            fn()
            n += 1
        out[name] = round(nbytes * n / (time.perf_counter() - t0) / 1e9, 3)
    return {"unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port", **out}


# --------------------------------------------------------------------------- distributed plumbing

def dist_setup(n_gpus: int) -> dict:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    ctx = {"world": world, "rank": rank, "local": local}
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        ctx["barrier"] = lambda: dist.barrier()

        def mx(v: float) -> float:
            t = torch.tensor([v], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        ctx["max"] = mx
    else:
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        ctx["barrier"] = lambda: None
        ctx["max"] = lambda v: v
    return ctx


def dist_teardown(ctx):
    if ctx["world"] > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


# --------------------------------------------------------------------------- main

def run_reference(args, ctx) -> None:
    if ctx["rank"] != 0:
        return
    from oracle import nki_oracle as O

    torch.set_num_threads(os.cpu_count() or 1)  # torchrun sets OMP_NUM_THREADS=1; use every host core
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(H, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
    t0 = time.perf_counter()
    for _ in range(min(args.warmup, 2)):
        O.attention_flash(q, k, v)
    per_step = (time.perf_counter() - t0) / max(1, min(args.warmup, 2))
    steps = max(1, min(args.steps, int(120.0 / max(per_step, 1e-3))))  # keep the arm within ~2 minutes
    t0 = time.perf_counter()
    for _ in range(steps):
        O.attention_flash(q, k, v)
    el = time.perf_counter() - t0
    val = ATTN_FLOP * steps / el / 1e12
    line = {"metric": METRIC, "value": round(val, 6), "unit": "TFLOPS", "n_gpus": args.gpus, "steps": steps,
            "warmup": args.warmup, "ms_per_step": round(el / steps * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
            "config": {"workload": "causal attention 8x2048x128 bf16 (BASELINE configs[3]) on host cores",
                       "heads": H, "seq_len": S, "head_dim": D},
            "cpu_baseline": {"value": round(val, 6), "unit": "TFLOPS", "cores": torch.get_num_threads(),
                             "kind": "port",
                             "sample": f"{steps} full steps of the CPU port of flash_attention_pipelined "
                                       "(the NKI simulator, the reference's own CPU path, is not installable here)"},
            "e2e": {"value": round(val, 6), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args, ctx) -> None:
    from nkilab import _native, ops  # noqa: F401  (loads the CUDA library, registers the ops)

    dev = torch.device("cuda", ctx["local"])
    world = ctx["world"]
    pk = peaks()
    stream = torch.cuda.Stream(dev)
    extra_err = {}
    # End to end through the public API first, in a process that has run nothing else yet:
    # after the large tensor-parallel block, the host round trips of later calls measured
    # 5-15 ms per step instead of 0.3-0.5 ms.
    e2e = bench_e2e(max(10, min(args.steps, 50)), args.warmup, dev, ctx)
    parity = sharded_parity(dev, ctx) if world > 1 else None
    with ClockSampler(ctx["local"]) as clk:
        from nkilab import parallel as P

        gather = P.preferred_gather(world)
        other = "nccl" if gather == "nvlink" else "nvlink"
        att = bench_attention_sharded(args.steps, args.warmup, dev, stream, ctx, gather=gather)
        att_other = bench_attention_sharded(args.steps, args.warmup, dev, stream, ctx, gather=other) if world > 1 else None
        rep = bench_attention(args.steps, args.warmup, dev, stream, ctx) if world > 1 else None
        rows = gemm = block = ladder = None
        if not args.headline_only:
            if world == 1:
                try:
                    ladder = bench_ladder(dev, stream, pk)
                except Exception as e:
                    extra_err["ladder"] = repr(e)
            try:
                rows = bench_rows(200, 5, dev, stream, pk)
            except Exception as e:  # report, keep the headline
                extra_err["row_kernels"] = repr(e)
            try:
                gemm = bench_gemm(dev, stream, pk)
            except Exception as e:
                extra_err["gemm"] = repr(e)
            try:
                block = bench_block(dev, stream, pk, ctx)
            except Exception as e:
                extra_err["decoder_block"] = repr(e)
    clocks = clk.summary()
    _native.check_device(torch.cuda.current_stream(dev).cuda_stream)
    e2e_val = ctx["max"](e2e["ms_per_step"])
    e2e["value"] = round(ATTN_FLOP / (e2e_val * 1e-3) / 1e12, 3)
    cpu = cpu_attention_baseline() if (ctx["rank"] == 0 and world == 1 and not args.no_cpu) else None
    cpu_rows = cpu_rows_baseline() if (cpu is not None) else None
    if ctx["rank"] != 0:
        return
    ms = att["ms_per_step"]
    value = ATTN_FLOP / (ms * 1e-3) / 1e12  # the whole 8-head job, all ranks together
    per_gpu = value / world
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "causal attention 8x2048x128 bf16, scale 1/sqrt(128) (BASELINE configs[3])",
                   "heads": H, "seq_len": S, "head_dim": D, "batch": 1,
                   "parallelism": (f"heads sharded over {world} GPUs ({att['heads_per_rank']} per rank); the output "
                                   + ("gathered to every rank over NVLink by the attention kernels"
                                      if gather == "nvlink" else "gathered to every rank by an NCCL all-gather")
                                   + " in the timed region (parallel.preferred_gather)")
                   if world > 1 else "single",
                   "l2": f"rotating pool of {att['pool_sets']} input sets, {att['pool_mib']:.0f} MiB > 2x L2",
                   "launch": "K steps in one CUDA graph via torch.ops.nkilab.attention (+ all-gather)"},
        "roofline": {"bound": "tensor", "achieved": round(per_gpu, 2), "peak": pk["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(per_gpu / pk["bf16_tflops"], 4),
                     "traffic": ncu_traffic("attn_fwd_bf16_8x2048x128.md") if world == 1 else None,
                     "algorithmic_flop_per_launch": ATTN_FLOP / world, "peak_source": pk["source"] + " burst bf16",
                     "kernel": "attn_fwd_bf16_kernel<128>",
                     "timed_over": "the whole op per step (attention kernel + split-KV combine kernel"
                                   + ((" + the NVLink gather and flag exchange" if gather == "nvlink"
                                       else " + the NCCL all-gather") if world > 1 else "")
                                   + "), per GPU, so 'achieved' is a lower bound for the attention kernel alone"},
        "clocks": clocks,
        "e2e": e2e,
        "gpu_launches": args.steps * att["launches_per_step"],
        "step_us_spread": att["us_per_step_rank0"],
    }
    if world > 1:
        what = {"nvlink": "attention kernels store every output tile into every rank's buffer over NVLink "
                          "(parallel.PeerAttention), then a flag exchange",
                "nccl": "NCCL all-gather of the output after the attention kernels"}
        line["sharded"] = {"gather": what[gather], "attention_us": att["attention_us"],
                           "gather_us": att["all_gather_us"], "heads_per_rank": att["heads_per_rank"],
                           "parity": parity,
                           f"{other}_gather_instead": {"us_per_step": round(att_other["ms_per_step"] * 1e3, 3),
                                                       "gather_us": att_other["all_gather_us"]}}
        rms = rep["ms_per_step"]
        line["replicas"] = {"value": round(ATTN_FLOP * world / (rms * 1e-3) / 1e12, 2), "unit": "TFLOPS",
                            "ms_per_step": round(rms, 5), "scaling": "weak",
                            "what": f"{world} independent 8x2048x128 problems, one per GPU, no collective"}
    if rows:
        line["row_kernels"] = {**rows, "peak_gbs": pk["hbm_gbs"], "peak_source": pk["source"],
                               "scope": "per GPU"}
    if gemm:
        line["gemm"] = gemm
    if block:
        line["decoder_block"] = block
    if ladder:
        line["ladder"] = ladder
    if cpu:
        line["cpu_baseline"] = cpu
        line["cpu_baseline_rows"] = cpu_rows
    if extra_err:
        line["errors"] = extra_err
    print(json.dumps(line), flush=True)


PROFILE_CASES = ("rmsnorm", "softmax", "swiglu", "gemm1024", "gemm8192", "attention", "attention_two_tile",
                 "attention_two_groups")


def run_profile_case(case: str, launches: int, rows: int = ROWS) -> None:
    """Launch one kernel `launches` times, eagerly and without timing, on BASELINE-shaped
    inputs, for an ncu capture (-k, -c). `rows` sets the row count of the row-kernel
    cases: a [4096, 2048] output (16.8 MB) stays in L2 when ncu times a single launch, so
    the write traffic shows only with more rows than L2 holds."""
    import ctypes

    from nkilab import _native as N

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    st = torch.cuda.current_stream(dev).cuda_stream
    bf = torch.bfloat16
    if case in ("rmsnorm", "softmax", "swiglu"):
        x, u = (torch.randn(rows, COLS, device=dev, generator=g).to(bf) for _ in range(2))
        w = (1 + 0.1 * torch.randn(COLS, device=dev, generator=g)).to(bf)
        y = torch.empty_like(x)
        for _ in range(launches):
            if case == "rmsnorm":
                N.call("nkl_rmsnorm", x.data_ptr(), w.data_ptr(), y.data_ptr(), rows, COLS, 1e-6, N.BFLOAT16, st)
            elif case == "softmax":
                N.call("nkl_softmax", x.data_ptr(), y.data_ptr(), rows, COLS, N.BFLOAT16, st)
            else:
                N.call("nkl_swiglu", x.data_ptr(), u.data_ptr(), y.data_ptr(), rows, COLS, N.BFLOAT16, st)
    elif case.startswith("gemm"):
        n = int(case[4:])
        a, b = ((torch.rand(n, n, device=dev, generator=g) * 2 - 1).to(bf) for _ in range(2))
        c = torch.empty(n, n, device=dev, dtype=bf)
        for _ in range(launches):
            N.call("nkl_matmul", a.data_ptr(), b.data_ptr(), c.data_ptr(), n, n, n, N.BFLOAT16, st)
    else:
        q, k, v = (torch.randn(H, S, D, device=dev, generator=g).to(bf) for _ in range(3))
        o = torch.empty_like(q)
        mode = {"attention_two_tile": N.ATTN_TWO_TILE, "attention_two_groups": N.ATTN_TWO_GROUPS}.get(case, N.ATTN_AUTO)
        nbytes = N.lib.nkl_attention_mode_workspace_size(H, S, D, N.BFLOAT16, mode)
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
        for _ in range(launches):
            N.call("nkl_attention_mode", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), ws.data_ptr(), nbytes,
                   H, S, D, 1.0 / math.sqrt(D), N.BFLOAT16, mode, st)
    torch.cuda.synchronize()
    N.check_device(st)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--headline-only", action="store_true", help="only the attention headline (for profiling)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--profile", choices=PROFILE_CASES,
                    help="only launch this kernel --steps times (untimed), for an ncu capture")
    ap.add_argument("--rows", type=int, default=ROWS, help="row count of the --profile row-kernel cases")
    args = ap.parse_args()
    if args.profile:
        from nkilab import ops  # noqa: F401  (loads the library)

        run_profile_case(args.profile, args.steps, args.rows)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        ctx = {"world": int(os.environ.get("WORLD_SIZE", "1")), "rank": int(os.environ.get("RANK", "0"))}
        run_reference(args, ctx)
        return
    ctx = dist_setup(args.gpus)
    try:
        run_ours(args, ctx)
    finally:
        dist_teardown(ctx)


if __name__ == "__main__":
    main()

"""Measured B200 results in the layout of the reference's dashboard data.

`python -m nkilab.results --out results.json [--quick]` times every kernel variant of
the reference's ladder on the GPU (warm-up, then the calls in one CUDA graph timed with
CUDA events; rotating inputs larger than L2) and writes a JSON file with the keys of the reference's
`site/data/results.json` (`bench/run_bench.py:238-258`: generated_at, git_sha, quick,
versions, hardware_model, matmul, norm, attention, decoder_block, correctness), so its
dashboard could render B200 data. The reference's `modeled_*` fields hold simulator
estimates; here they hold the measured values, and `measured: true` says so. Inputs
rotate through sets larger than L2; outputs come from the graph's memory pool and may
reuse one buffer, so the memory-bound rows read like a warm-output figure (bench.py's
row-kernel section rotates outputs too and is the conservative number).
"""
from __future__ import annotations

import argparse
import datetime as dt
import json
import math
import os
import platform
import subprocess

import numpy as np
import torch

from . import _torch_ops, model, ops  # noqa: F401  (registers torch.ops.nkilab.*)

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
_L2_BYTES = 126 << 20


def _peaks() -> dict:
    try:
        with open(os.path.join(_ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_bytes_per_s": float(p["hbm_gbs"]) * 1e9, "bf16_flops": float(p["bf16_tflops"]) * 1e12,
                "source": "measured (MEASURED_PEAKS.json)"}
    except (OSError, KeyError, ValueError):
        return {"hbm_bytes_per_s": 6.65e12, "bf16_flops": 1.59e15, "source": "fallback"}


def _time_us(step, reps: int) -> float:
    """Mean device time of step(i) over `reps` calls: warm-up, then the calls captured in
    one CUDA graph (so host launch overhead does not pace the GPU), one untimed replay,
    one replay timed with CUDA events."""
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(3):
            step(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(reps):
            step(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / reps


def _entry(kernel: str, us: float, hbm_bytes: int, flops: int, pk: dict, dtype_flops: float) -> dict:
    mem_us = hbm_bytes / pk["hbm_bytes_per_s"] * 1e6
    cmp_us = flops / dtype_flops * 1e6 if flops else 0.0
    bound = max(mem_us, cmp_us)
    return {"kernel": kernel, "measured": True, "hbm_bytes": int(hbm_bytes), "flops": int(flops),
            "measured_latency_us": round(us, 3), "modeled_latency_us": round(us, 3),
            "roofline_bound_us": round(bound, 3), "roofline_regime": "compute" if cmp_us > mem_us else "memory",
            "arithmetic_intensity": (flops / hbm_bytes) if hbm_bytes else 0.0,
            "measured_tflops": round(flops / (us * 1e-6) / 1e12, 3) if flops else 0.0,
            "modeled_tflops": round(flops / (us * 1e-6) / 1e12, 3) if flops else 0.0,
            "achieved_gbs": round(hbm_bytes / (us * 1e-6) / 1e9, 1),
            "pct_of_roofline": round(100.0 * bound / us, 2)}


def _rotating(make, bytes_per_set: int) -> list:
    return [make() for _ in range(max(2, math.ceil(2 * _L2_BYTES / max(1, bytes_per_set))))]


def bench_matmul(pk: dict, quick: bool) -> dict:
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)

    def mats(n):
        return [(torch.rand(n, n, device=dev, generator=g) * 2 - 1).to(torch.bfloat16) for _ in range(2)]

    n = 1024
    sets = _rotating(lambda: mats(n), 3 * n * n * 2)
    variants = []
    for name, variant in (("matmul naive", "naive"), ("matmul blocked (TMA + tcgen05)", "blocked")):
        us = _time_us(lambda i: torch.ops.nkilab.matmul(*sets[i % len(sets)], variant == "naive"), 10 if quick else 30)
        variants.append(_entry(name, us, 3 * n * n * 2, 2 * n ** 3, pk, pk["bf16_flops"]))
    sweep = []
    for m in ([512, 1024, 2048] if quick else [512, 1024, 2048, 4096, 8192]):
        sm = _rotating(lambda: mats(m), 3 * m * m * 2) if m <= 4096 else [mats(m)]
        for variant in (["naive", "blocked"] if m <= 2048 else ["blocked"]):
            us = _time_us(lambda i: torch.ops.nkilab.matmul(*sm[i % len(sm)], variant == "naive"), 5 if m >= 4096 else 20)
            e = _entry(f"matmul {variant}", us, 3 * m * m * 2, 2 * m ** 3, pk, pk["bf16_flops"])
            sweep.append({"n": m, "variant": variant, "modeled_latency_us": e["modeled_latency_us"],
                          "measured_latency_us": e["measured_latency_us"], "hbm_bytes": e["hbm_bytes"],
                          "flops": e["flops"], "arithmetic_intensity": e["arithmetic_intensity"],
                          "modeled_tflops": e["modeled_tflops"], "ideal_bound_us": e["roofline_bound_us"]})
        del sm
    return {"shape": [n, n, n], "dtype": "bfloat16", "variants": variants, "sweep": sweep}


def bench_norm(pk: dict, quick: bool) -> dict:
    dev = "cuda"
    R, C = 4096, 2048
    g = torch.Generator(device=dev).manual_seed(1)
    xb = R * C * 2
    reps = 20 if quick else 100
    sets = _rotating(lambda: [torch.randn(R, C, device=dev, generator=g).to(torch.bfloat16) for _ in range(2)], 4 * xb)
    w = (1 + 0.1 * torch.randn(C, device=dev, generator=g)).to(torch.bfloat16)
    cases = [
        ("softmax unfused (3 HBM passes)", lambda i: torch.ops.nkilab.softmax(sets[i % len(sets)][0], False),
         2 * xb + 3 * R * C * 4 + 2 * R * 4),
        ("softmax fused", lambda i: torch.ops.nkilab.softmax(sets[i % len(sets)][0], True), 2 * xb),
        ("rmsnorm fused", lambda i: torch.ops.nkilab.rmsnorm(sets[i % len(sets)][0], w, 1e-6), 2 * xb + C * 2),
        ("residual add + rmsnorm fused",
         lambda i: torch.ops.nkilab.add_rmsnorm(sets[i % len(sets)][0], sets[i % len(sets)][1], w, 1e-6),
         4 * xb + C * 2),
        ("swiglu fused", lambda i: torch.ops.nkilab.swiglu(sets[i % len(sets)][0], sets[i % len(sets)][1]), 3 * xb),
    ]
    variants = [_entry(name, _time_us(fn, reps), nbytes, 0, pk, pk["bf16_flops"]) for name, fn, nbytes in cases]
    return {"shape": [R, C], "dtype": "bfloat16", "variants": variants}


def bench_attention(pk: dict, quick: bool) -> dict:
    dev = "cuda"
    H, S, D = 8, 2048, 128
    g = torch.Generator(device=dev).manual_seed(2)

    def qkv(h, s):
        return [torch.randn(h, s, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(3)]

    flops = 2 * H * S * S * D
    io = 4 * H * S * D * 2
    sets = _rotating(lambda: qkv(H, S), io)
    scale = 1.0 / math.sqrt(D)
    ladder = []
    naive_bytes = io + H * S * S * (4 + 2) * 2  # scores (fp32) and probabilities (bf16) written and read back
    us = _time_us(lambda i: torch.ops.nkilab.attention(*sets[i % len(sets)], scale, True), 5 if quick else 20)
    ladder.append(_entry("naive (scores in HBM)", us, naive_bytes, flops, pk, pk["bf16_flops"]))
    us_flash = _time_us(lambda i: torch.ops.nkilab.attention(*sets[i % len(sets)], scale, False), 20 if quick else 100)
    for name in ("flash", "flash kv_resident", "flash balanced", "flash pipelined"):
        e = _entry(f"{name} (one tcgen05 kernel for every flash variant)", us_flash, io, flops, pk, pk["bf16_flops"])
        ladder.append(e)
    scaling = []
    for s in ([512, 1024, 2048] if quick else [512, 1024, 2048, 4096]):
        sc = _rotating(lambda: qkv(H, s), 4 * H * s * D * 2)
        for variant in ("naive", "flash"):
            if variant == "naive" and s > 2048:
                continue
            us = _time_us(lambda i: torch.ops.nkilab.attention(*sc[i % len(sc)], scale, variant == "naive"), 10)
            hb = 4 * H * s * D * 2 + (H * s * s * 12 if variant == "naive" else 0)
            scaling.append({"S": s, "variant": variant, "hbm_bytes": hb, "measured_latency_us": round(us, 3),
                            "modeled_latency_us": round(us, 3),
                            "measured_tflops": round(2 * H * s * s * D / (us * 1e-6) / 1e12, 3)})
        del sc
    return {"shape": [H, S, D], "dtype": "bfloat16", "ladder": ladder, "scaling": scaling}


def bench_block(pk: dict, quick: bool) -> dict:
    """The reference's block configuration (fp32, S=512, d=256): error of the device
    forward against the torch module, and every stage timed on its own."""
    torch.manual_seed(0)
    cfg = model.BlockConfig(d_model=256, n_heads=4, d_ff=1024)
    block = model.DecoderBlock(cfg)
    S, d, H, hd = 512, cfg.d_model, cfg.n_heads, cfg.head_dim
    x = torch.randn(S, d)
    with torch.no_grad():
        ref = block(x)
    got = model.nki_forward(block, x.cuda()).cpu()
    w = model.device_weights(block, torch.float32, torch.device("cuda"))
    xd = x.cuda()
    h = ops.rmsnorm(xd, w["norm1"], cfg.eps)
    qkv = ops.matmul(h, w["wqkv"])
    q, k, v = (qkv[:, i * d:(i + 1) * d].reshape(S, H, hd).transpose(0, 1).contiguous() for i in range(3))
    att = ops.attention(q, k, v).transpose(0, 1).reshape(S, d).contiguous()
    proj = ops.matmul(att, w["wo"])
    x1, h2 = torch.ops.nkilab.add_rmsnorm(xd, proj, w["norm2"], cfg.eps)
    gt, up = ops.matmul(h2, w["wg"]), ops.matmul(h2, w["wu"])
    act = ops.swiglu(gt, up)
    f4 = 4  # fp32 bytes
    stages = [
        ("rmsnorm", lambda i: ops.rmsnorm(xd, w["norm1"], cfg.eps), 2 * S * d * f4, 0),
        ("matmul qkv", lambda i: ops.matmul(h, w["wqkv"]), (S * d + 3 * d * d + 3 * S * d) * f4, 6 * S * d * d),
        ("attention", lambda i: ops.attention(q, k, v), 4 * S * d * f4, 2 * H * S * S * hd),
        ("matmul wo", lambda i: ops.matmul(att, w["wo"]), (2 * S * d + d * d) * f4, 2 * S * d * d),
        ("residual add + rmsnorm", lambda i: torch.ops.nkilab.add_rmsnorm(xd, proj, w["norm2"], cfg.eps),
         4 * S * d * f4, 0),
        ("matmul gate + up", lambda i: (ops.matmul(h2, w["wg"]), ops.matmul(h2, w["wu"])),
         2 * (S * d + d * cfg.d_ff + S * cfg.d_ff) * f4, 4 * S * d * cfg.d_ff),
        ("swiglu", lambda i: ops.swiglu(gt, up), 3 * S * cfg.d_ff * f4, 0),
        ("matmul down", lambda i: ops.matmul(act, w["wd"]), (S * cfg.d_ff + cfg.d_ff * d + S * d) * f4,
         2 * S * cfg.d_ff * d),
    ]
    parts = []
    for op, fn, nbytes, fl in stages:
        us = _time_us(fn, 20)
        parts.append({"op": op, "measured_latency_us": round(us, 3), "modeled_latency_us": round(us, 3),
                      "hbm_bytes": nbytes, "flops": fl})
    del x1
    return {"config": {"d_model": d, "n_heads": H, "d_ff": cfg.d_ff, "eps": cfg.eps}, "seq_len": S,
            "dtype": "float32", "max_abs_err_vs_pytorch": float((got - ref).abs().max()),
            "max_abs_ref": float(ref.abs().max()), "parts": parts}


def correctness() -> list:
    out = []
    g = torch.Generator().manual_seed(3)
    x = torch.randn(300, 777, generator=g)
    out.append({"op": "softmax fused", "shape": "300x777",
                "vs_torch": float((ops.softmax(x.cuda()).cpu() - torch.softmax(x, -1)).abs().max())})
    w = 1 + 0.1 * torch.randn(777, generator=g)
    ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    out.append({"op": "rmsnorm fused", "shape": "300x777",
                "vs_torch": float((ops.rmsnorm(x.cuda(), w.cuda(), 1e-6).cpu() - ref).abs().max())})
    u = torch.randn(300, 777, generator=g)
    out.append({"op": "swiglu fused", "shape": "300x777",
                "vs_torch": float((ops.swiglu(x.cuda(), u.cuda()).cpu() - torch.nn.functional.silu(x) * u).abs().max())})
    a, b = torch.randn(200, 300, generator=g), torch.randn(300, 130, generator=g)
    out.append({"op": "matmul blocked", "shape": "200x300x130",
                "vs_torch": float((ops.matmul(a.cuda(), b.cuda()).cpu() - a @ b).abs().max())})
    q, k, v = (torch.randn(2, 300, 64, generator=g) for _ in range(3))
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
    for variant in ("naive", "flash_pipelined"):
        out.append({"op": f"attention {variant}", "shape": "2x300x64",
                    "vs_torch": float((ops.attention(q.cuda(), k.cuda(), v.cuda(), variant).cpu() - ref).abs().max())})
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--out", default="results.json")
    ap.add_argument("--quick", action="store_true")
    a = ap.parse_args(argv)
    pk = _peaks()
    try:
        sha = subprocess.run(["git", "rev-parse", "--short", "HEAD"], capture_output=True, text=True,
                             cwd=_ROOT).stdout.strip()
    except OSError:
        sha = ""
    props = torch.cuda.get_device_properties(0)
    result = {
        "generated_at": dt.datetime.now(dt.timezone.utc).isoformat(timespec="seconds"),
        "git_sha": sha, "quick": a.quick,
        "versions": {"python": platform.python_version(), "torch": torch.__version__,
                     "cuda": torch.version.cuda or "", "numpy": np.__version__},
        "hardware_model": {"name": f"{props.name} (sm_{props.major}{props.minor}a)",
                           "sms": props.multi_processor_count, "hbm_bytes": props.total_memory,
                           "hbm_bytes_per_s": pk["hbm_bytes_per_s"], "peak_flops": {"bfloat16": pk["bf16_flops"]},
                           "peaks_source": pk["source"]},
        "matmul": bench_matmul(pk, a.quick), "norm": bench_norm(pk, a.quick),
        "attention": bench_attention(pk, a.quick), "decoder_block": bench_block(pk, a.quick),
        "correctness": correctness(),
    }
    with open(a.out, "w") as f:
        json.dump(result, f, indent=1, default=float)
    print("wrote", os.path.abspath(a.out))


if __name__ == "__main__":
    main()

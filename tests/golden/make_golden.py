"""Generate the golden vectors in this directory from the reference's own code.

    python tests/golden/make_golden.py --reference PATH   (or NKL_REFERENCE=PATH in the environment)

PATH is a checkout of Nags-gk/nki-kernel-lab.

Runs the unmodified Nags-gk/nki-kernel-lab sources -- nkilab/ops.py host wrappers,
nkilab/kernels/*.py NKI kernels and nkilab/model.py -- with nki_shim.py standing in
for the ``nki`` package (not installable here), on small seeded inputs shaped like
the reference's tests (tests/test_*.py), and stores inputs and outputs:

    golden_attention.npz  every ATTENTION_VARIANTS entry on fp32 / bf16 cases
    golden_matmul.npz     ops.matmul blocked + naive, fp32 / bf16, odd shapes
    golden_norm.npz       ops.softmax (fused, unfused), ops.rmsnorm, ops.swiglu
    golden_model.npz      model.nki_forward and DecoderBlock.forward, fp32 / bf16
    golden_blocks.json    ops.choose_blocks over a grid of tile counts

bf16 arrays are stored as their uint16 bit patterns under keys ending in "@bf16".
The reference tree is read, never written; nothing at test time needs it.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import ml_dtypes
import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BF16 = ml_dtypes.bfloat16


def put(store: dict, key: str, arr) -> None:
    arr = np.asarray(arr)
    if arr.dtype == BF16:
        store[key + "@bf16"] = arr.view(np.uint16)
    else:
        store[key] = arr


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("NKL_REFERENCE"),
                    help="checkout of Nags-gk/nki-kernel-lab (default: $NKL_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference PATH or set NKL_REFERENCE")

    sys.path.insert(0, HERE)
    import nki_shim

    nki_shim.install()
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch
    from nkilab import ops  # the reference's host wrappers, running on the shim
    from nkilab.model import BlockConfig, DecoderBlock, nki_forward

    # ------------------------------------------------------------------ attention
    att = {}
    cases = [
        ("f32_1_128_64", np.float32, (1, 128, 64), list(ops.ATTENTION_VARIANTS)),
        ("f32_2_200_32", np.float32, (2, 200, 32), list(ops.ATTENTION_VARIANTS)),
        ("f32_1_384_128", np.float32, (1, 384, 128), ["naive", "flash_pipelined"]),
        ("bf16_2_256_64", BF16, (2, 256, 64), ["naive", "flash", "flash_pipelined"]),
        ("bf16_1_300_128", BF16, (1, 300, 128), ["naive", "flash_pipelined"]),
    ]
    for i, (name, dt, shape, variants) in enumerate(cases):
        rng = np.random.default_rng(1000 + i)
        q, k, v = (rng.standard_normal(shape).astype(dt) for _ in range(3))
        put(att, f"{name}/q", q)
        put(att, f"{name}/k", k)
        put(att, f"{name}/v", v)
        for var in variants:
            put(att, f"{name}/out_{var}", ops.attention(q, k, v, variant=var))
        print("attention", name, variants, flush=True)
    np.savez_compressed(os.path.join(HERE, "golden_attention.npz"), **att)

    # ------------------------------------------------------------------ matmul
    mm = {}
    cases = [
        ("f32_128_128_512", np.float32, (128, 128, 512), "normal"),
        ("f32_200_300_130", np.float32, (200, 300, 130), "normal"),
        ("f32_1_7_3", np.float32, (1, 7, 3), "normal"),
        ("bf16_128_512_256", BF16, (128, 512, 256), "normal"),
        ("bf16_200_300_130", BF16, (200, 300, 130), "uniform"),
    ]
    for i, (name, dt, (M, K, N), dist) in enumerate(cases):
        rng = np.random.default_rng(2000 + i)
        if dist == "normal":
            a = rng.standard_normal((M, K)).astype(dt)
            b = rng.standard_normal((K, N)).astype(dt)
        else:
            a = rng.uniform(-1, 1, (M, K)).astype(dt)
            b = rng.uniform(-1, 1, (K, N)).astype(dt)
        put(mm, f"{name}/a", a)
        put(mm, f"{name}/b", b)
        for var in ("blocked", "naive"):
            put(mm, f"{name}/out_{var}", ops.matmul(a, b, variant=var))
        print("matmul", name, flush=True)
    np.savez_compressed(os.path.join(HERE, "golden_matmul.npz"), **mm)

    # ------------------------------------------------------------------ row kernels
    nm = {}
    sm_cases = [("f32_128_64", np.float32, (128, 64), 4.0), ("f32_5_3", np.float32, (5, 3), 4.0),
                ("f32_40_1024", np.float32, (40, 1024), 4.0), ("f32_64_512_big", np.float32, (64, 512), 1e4),
                ("bf16_256_512", BF16, (256, 512), 1.0)]
    for i, (name, dt, shape, scale) in enumerate(sm_cases):
        rng = np.random.default_rng(3000 + i)
        x = (rng.standard_normal(shape) * scale).astype(dt)
        put(nm, f"softmax_{name}/x", x)
        put(nm, f"softmax_{name}/out_fused", ops.softmax(x, fused=True))
        put(nm, f"softmax_{name}/out_unfused", ops.softmax(x, fused=False))
    rms_cases = [("f32_7_33", np.float32, (7, 33), "uniform"), ("f32_40_1024", np.float32, (40, 1024), "uniform"),
                 ("bf16_256_512_ones", BF16, (256, 512), "ones"), ("bf16_32_2048", BF16, (32, 2048), "normal")]
    for i, (name, dt, (R, D), wdist) in enumerate(rms_cases):
        rng = np.random.default_rng(4000 + i)
        x = rng.standard_normal((R, D)).astype(dt)
        if wdist == "uniform":
            w = rng.uniform(0.5, 1.5, D).astype(dt)
        elif wdist == "ones":
            w = np.ones(D, dt)
        else:
            w = (1.0 + 0.1 * rng.standard_normal(D)).astype(dt)
        put(nm, f"rmsnorm_{name}/x", x)
        put(nm, f"rmsnorm_{name}/w", w)
        put(nm, f"rmsnorm_{name}/out", ops.rmsnorm(x, w))
    sw_cases = [("f32_32_1024", np.float32, (32, 1024)), ("f32_7_33", np.float32, (7, 33)),
                ("bf16_128_512", BF16, (128, 512))]
    for i, (name, dt, shape) in enumerate(sw_cases):
        rng = np.random.default_rng(5000 + i)
        g = rng.standard_normal(shape).astype(dt)
        u = rng.standard_normal(shape).astype(dt)
        put(nm, f"swiglu_{name}/gate", g)
        put(nm, f"swiglu_{name}/up", u)
        put(nm, f"swiglu_{name}/out", ops.swiglu(g, u))
    print("norm done", flush=True)
    np.savez_compressed(os.path.join(HERE, "golden_norm.npz"), **nm)

    # ------------------------------------------------------------------ decoder block
    md = {}
    for name, S, dt, variant in [("f32_128_flash", 128, np.float32, "flash_pipelined"),
                                 ("f32_300_naive", 300, np.float32, "naive"),
                                 ("bf16_128_flash", 128, BF16, "flash_pipelined")]:
        torch.manual_seed(0)
        block = DecoderBlock(BlockConfig()).eval()
        x = torch.randn(S, block.cfg.d_model)
        with torch.no_grad():
            ref = block(x).numpy()
        xin = x.numpy().astype(dt)
        out = nki_forward(block, xin, attention_variant=variant)
        put(md, f"{name}/x", xin)
        put(md, f"{name}/out_nki_forward", out)
        md[f"{name}/out_torch_block"] = ref
        md[f"{name}/param_sums"] = np.array([p.detach().double().sum().item() for p in block.parameters()])
        print("model", name, flush=True)
    np.savez_compressed(os.path.join(HERE, "golden_model.npz"), **md)

    table = {f"{m},{n}": list(ops.choose_blocks(m, n)) for m in range(1, 9) for n in range(1, 17)}
    with open(os.path.join(HERE, "golden_blocks.json"), "w") as f:
        json.dump(table, f, indent=0, sort_keys=True)
    print("done")


if __name__ == "__main__":
    main()

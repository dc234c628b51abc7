"""PyTorch custom ops (namespace ``nkilab``) over the C ABI.

Each op takes contiguous CUDA tensors, allocates its output with the caching
allocator, and launches the C-ABI entry point on the current CUDA stream, so the ops
compose with streams and CUDA-graph capture like any torch op:

    torch.ops.nkilab.rmsnorm(x, weight, eps)        -> nkl_rmsnorm
    torch.ops.nkilab.softmax(x, fused)              -> nkl_softmax / nkl_softmax_unfused
    torch.ops.nkilab.swiglu(gate, up)               -> nkl_swiglu
    torch.ops.nkilab.matmul(a, b, naive)            -> nkl_matmul / nkl_matmul_naive
    torch.ops.nkilab.matmul_f32out(a, b)            -> nkl_matmul_f32out (bf16 in, fp32 out)
    torch.ops.nkilab.attention(q, k, v, scale, naive) -> nkl_attention_ws / nkl_attention_naive

There is no CPU implementation: a CPU tensor is an error, never a fallback.
"""
from __future__ import annotations

import torch

from . import _native as N

_DTYPES = {torch.float32: N.FLOAT32, torch.bfloat16: N.BFLOAT16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"nkilab kernels support float32 and bfloat16, got {t.dtype}") from None


def _prep(*ts: torch.Tensor):
    dev = ts[0].device
    if dev.type != "cuda":
        raise RuntimeError("nkilab ops run on CUDA tensors only (no CPU implementation)")
    for t in ts:
        if t.device != dev:
            raise RuntimeError(f"tensors on different devices: {t.device} vs {dev}")
        if t.dtype != ts[0].dtype:
            raise TypeError(f"mixed dtypes: {t.dtype} vs {ts[0].dtype}")
        if not t.is_contiguous():
            raise RuntimeError("nkilab ops need contiguous tensors")
    return dev, dtype_code(ts[0]), torch.cuda.current_stream(dev).cuda_stream


def _rows(x: torch.Tensor):
    cols = x.shape[-1] if x.dim() else 1
    rows = x.numel() // cols if cols else 0
    return rows, cols


@torch.library.custom_op("nkilab::rmsnorm", mutates_args=())
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    dev, dt, st = _prep(x, weight)
    rows, cols = _rows(x)
    if weight.numel() != cols:
        raise ValueError(f"weight has {weight.numel()} elements, rows have {cols}")
    out = torch.empty_like(x)
    with torch.cuda.device(dev):
        N.call("nkl_rmsnorm", x.data_ptr(), weight.data_ptr(), out.data_ptr(), rows, cols, eps, dt, st)
    return out


@rmsnorm.register_fake
def _(x, weight, eps):
    return torch.empty_like(x)


@torch.library.custom_op("nkilab::softmax", mutates_args=())
def softmax(x: torch.Tensor, fused: bool) -> torch.Tensor:
    dev, dt, st = _prep(x)
    rows, cols = _rows(x)
    out = torch.empty_like(x)
    with torch.cuda.device(dev):
        if fused:
            N.call("nkl_softmax", x.data_ptr(), out.data_ptr(), rows, cols, dt, st)
        else:
            nbytes = N.lib.nkl_softmax_unfused_workspace_size(rows, cols)
            ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
            N.call("nkl_softmax_unfused", x.data_ptr(), out.data_ptr(), ws.data_ptr(), nbytes, rows, cols, dt, st)
    return out


@softmax.register_fake
def _(x, fused):
    return torch.empty_like(x)


@torch.library.custom_op("nkilab::swiglu", mutates_args=())
def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    dev, dt, st = _prep(gate, up)
    if gate.shape != up.shape:
        raise ValueError(f"gate {tuple(gate.shape)} and up {tuple(up.shape)} differ")
    rows, cols = _rows(gate)
    out = torch.empty_like(gate)
    with torch.cuda.device(dev):
        N.call("nkl_swiglu", gate.data_ptr(), up.data_ptr(), out.data_ptr(), rows, cols, dt, st)
    return out


@swiglu.register_fake
def _(gate, up):
    return torch.empty_like(gate)


@torch.library.custom_op("nkilab::matmul", mutates_args=())
def matmul(a: torch.Tensor, b: torch.Tensor, naive: bool) -> torch.Tensor:
    dev, dt, st = _prep(a, b)
    M, K = a.shape
    K2, Ncols = b.shape
    if K != K2:
        raise ValueError(f"inner dimensions differ: {tuple(a.shape)} @ {tuple(b.shape)}")
    out = torch.empty((M, Ncols), dtype=a.dtype, device=dev)
    with torch.cuda.device(dev):
        fn = "nkl_matmul_naive" if naive else "nkl_matmul"
        N.call(fn, a.data_ptr(), b.data_ptr(), out.data_ptr(), M, Ncols, K, dt, st)
    return out


@matmul.register_fake
def _(a, b, naive):
    return a.new_empty((a.shape[0], b.shape[1]))


@torch.library.custom_op("nkilab::add_rmsnorm", mutates_args=())
def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(x + residual rounded to x.dtype, rmsnorm of that sum) in one pass."""
    dev, dt, st = _prep(x, residual, weight)
    if residual.shape != x.shape:
        raise ValueError(f"x {tuple(x.shape)} and residual {tuple(residual.shape)} must match")
    cols = x.shape[-1]
    rows = x.numel() // cols if cols else 0
    s = torch.empty_like(x)
    out = torch.empty_like(x)
    with torch.cuda.device(dev):
        N.call("nkl_add_rmsnorm", x.data_ptr(), residual.data_ptr(), weight.data_ptr(), s.data_ptr(), out.data_ptr(),
               rows, cols, eps, dt, st)
    return s, out


@add_rmsnorm.register_fake
def _(x, residual, weight, eps):
    return torch.empty_like(x), torch.empty_like(x)


@torch.library.custom_op("nkilab::rope", mutates_args=())
def rope(x: torch.Tensor, base: float, pos_offset: int) -> torch.Tensor:
    """Rotary position embedding (rotate-half) of x [heads, seq, head_dim]."""
    dev, dt, st = _prep(x)
    H, S, d = x.shape
    out = torch.empty_like(x)
    with torch.cuda.device(dev):
        N.call("nkl_rope", x.data_ptr(), out.data_ptr(), H, S, d, base, pos_offset, dt, st)
    return out


@rope.register_fake
def _(x, base, pos_offset):
    return torch.empty_like(x)


SWIGLU_BLOCK = 128  # column block of the interleaved [gate | up] weight of matmul_swiglu


def interleave_gate_up(wg: torch.Tensor, wu: torch.Tensor) -> torch.Tensor:
    """[K, F] gate and up weights -> the [K, 2F] layout nkl_matmul_swiglu reads: column
    blocks of 128, gate block i followed by up block i."""
    K, F = wg.shape
    if wu.shape != wg.shape or F % SWIGLU_BLOCK:
        raise ValueError(f"gate {tuple(wg.shape)} / up {tuple(wu.shape)}: need equal shapes and F % 128 == 0")
    g = wg.reshape(K, F // SWIGLU_BLOCK, 1, SWIGLU_BLOCK)
    u = wu.reshape(K, F // SWIGLU_BLOCK, 1, SWIGLU_BLOCK)
    return torch.cat([g, u], dim=2).reshape(K, 2 * F).contiguous()


@torch.library.custom_op("nkilab::matmul_swiglu", mutates_args=())
def matmul_swiglu(a: torch.Tensor, b_gate_up: torch.Tensor) -> torch.Tensor:
    """silu(a @ Wg) * (a @ Wu) in one GEMM over the interleaved weight (bf16)."""
    dev, dt, st = _prep(a, b_gate_up)
    M, K = a.shape
    K2, two_f = b_gate_up.shape
    if K != K2 or two_f % (2 * SWIGLU_BLOCK):
        raise ValueError(f"a {tuple(a.shape)}, b_gate_up {tuple(b_gate_up.shape)}: need matching K and 2F % 256 == 0")
    out = torch.empty((M, two_f // 2), dtype=a.dtype, device=dev)
    with torch.cuda.device(dev):
        N.call("nkl_matmul_swiglu", a.data_ptr(), b_gate_up.data_ptr(), out.data_ptr(), M, two_f // 2, K, dt, st)
    return out


@matmul_swiglu.register_fake
def _(a, b_gate_up):
    return a.new_empty((a.shape[0], b_gate_up.shape[1] // 2))


@torch.library.custom_op("nkilab::matmul_residual", mutates_args=())
def matmul_residual(a: torch.Tensor, b: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    """residual + a @ b with the add in the GEMM epilogue (bf16; same bits as matmul, then add)."""
    dev, dt, st = _prep(a, b, residual)
    M, K = a.shape
    K2, Ncols = b.shape
    if K != K2 or residual.shape != (M, Ncols):
        raise ValueError(f"a {tuple(a.shape)}, b {tuple(b.shape)}, residual {tuple(residual.shape)}: shapes do not match")
    out = torch.empty((M, Ncols), dtype=a.dtype, device=dev)
    with torch.cuda.device(dev):
        N.call("nkl_matmul_residual", a.data_ptr(), b.data_ptr(), residual.data_ptr(), out.data_ptr(), M, Ncols, K,
               dt, st)
    return out


@matmul_residual.register_fake
def _(a, b, residual):
    return a.new_empty((a.shape[0], b.shape[1]))


@torch.library.custom_op("nkilab::matmul_f32out", mutates_args=())
def matmul_f32out(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a @ b for bf16 a, b with the fp32 accumulator returned unrounded (float32 [M, N])."""
    dev, dt, st = _prep(a, b)
    M, K = a.shape
    K2, Ncols = b.shape
    if K != K2:
        raise ValueError(f"inner dimensions differ: {tuple(a.shape)} @ {tuple(b.shape)}")
    out = torch.empty((M, Ncols), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        N.call("nkl_matmul_f32out", a.data_ptr(), b.data_ptr(), out.data_ptr(), M, Ncols, K, dt, st)
    return out


@matmul_f32out.register_fake
def _(a, b):
    return a.new_empty((a.shape[0], b.shape[1]), dtype=torch.float32)


# Split-KV workspaces of the bf16 attention kernel. Eager calls share one workspace per
# (device, stream), grown on demand (the kernels need no initialised contents): calls on
# one stream are ordered, so they can share it, and other streams get their own. A call
# made while its stream is being captured into a CUDA graph takes a fresh workspace from
# the caching allocator instead, which during capture hands out memory of the graph's
# own pool: every graph then owns the workspaces it writes, two graphs can be replayed
# concurrently, and replacing an outgrown eager workspace never frees memory a graph
# still uses.
_attention_ws: dict = {}


def _attention_workspace(dev: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    if dev.type == "cuda" and torch.cuda.is_current_stream_capturing():
        return torch.empty(nbytes, dtype=torch.uint8, device=dev)
    key = (dev.index, stream)
    ws = _attention_ws.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        _attention_ws[key] = ws
    return ws


@torch.library.custom_op("nkilab::attention", mutates_args=())
def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, naive: bool) -> torch.Tensor:
    dev, dt, st = _prep(q, k, v)
    H, S, d = q.shape
    Hkv = k.shape[0]
    if k.shape != v.shape or k.shape[1:] != q.shape[1:] or Hkv < 1 or H % Hkv:
        raise ValueError(f"q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)}: k and v must match, "
                         "and their head count divide q's")
    if naive and Hkv != H:
        raise ValueError("the naive variant needs as many key/value heads as query heads")
    out = torch.empty_like(q)
    with torch.cuda.device(dev):
        if Hkv != H:  # grouped-query / multi-query attention
            nbytes = N.lib.nkl_attention_workspace_size(H, S, d, dt)
            ws = _attention_workspace(dev, st, nbytes) if nbytes else None
            N.call("nkl_attention_gqa", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                   ws.data_ptr() if ws is not None else None, nbytes, H, Hkv, S, d, scale, dt, st)
        elif naive:
            nbytes = N.lib.nkl_attention_naive_workspace_size(H, S, dt)
            ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
            N.call("nkl_attention_naive", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), ws.data_ptr(),
                   nbytes, H, S, d, scale, dt, st)
        else:
            nbytes = N.lib.nkl_attention_workspace_size(H, S, d, dt)
            if nbytes:
                ws = _attention_workspace(dev, st, nbytes)
                N.call("nkl_attention_ws", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), ws.data_ptr(),
                       nbytes, H, S, d, scale, dt, st)
            else:
                N.call("nkl_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), H, S, d, scale,
                       dt, st)
    return out


@attention.register_fake
def _(q, k, v, scale, naive):
    return torch.empty_like(q)


@torch.library.custom_op("nkilab::attention_strided_", mutates_args=("out",))
def attention_strided_(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, scale: float) -> None:
    """Causal attention into `out` for strided views: q and out [H, S, d], k and v
    [Hkv, S, d], each with unit stride along d and any head / seq strides that are
    multiples of 8 elements (k and v with equal strides), e.g. q = qkv[:, 0].transpose(0, 1)
    of a [S, 3, H, d] projection and out = o.view(S, H, d).transpose(0, 1). bf16 only."""
    dev = q.device
    for t in (k, v, out):
        if t.device != dev or t.dtype != q.dtype:
            raise RuntimeError("attention_strided_: tensors must share device and dtype")
    if dev.type != "cuda" or q.dtype != torch.bfloat16:
        raise RuntimeError("attention_strided_: bf16 CUDA tensors only")
    H, S, d = q.shape
    Hkv = k.shape[0]
    if (k.shape != v.shape or k.shape[1:] != q.shape[1:] or out.shape != q.shape or Hkv < 1 or H % Hkv
            or k.stride() != v.stride() or any(t.stride(2) != 1 for t in (q, k, v, out))):
        raise ValueError(f"q {tuple(q.shape)}/{q.stride()}, k {tuple(k.shape)}/{k.stride()}, "
                         f"v {tuple(v.shape)}/{v.stride()}, out {tuple(out.shape)}/{out.stride()}: bad layout")
    dt = dtype_code(q)
    st = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        nbytes = N.lib.nkl_attention_workspace_size(H, S, d, dt)
        ws = _attention_workspace(dev, st, nbytes) if nbytes else None
        N.call("nkl_attention_strided", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
               ws.data_ptr() if ws is not None else None, nbytes, H, Hkv, S, d, q.stride(1), q.stride(0),
               k.stride(1), k.stride(0), out.stride(1), out.stride(0), scale, dt, st)


@attention_strided_.register_fake
def _(q, k, v, out, scale):
    return None

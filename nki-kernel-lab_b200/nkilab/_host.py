"""Host <-> device conversion shared by nkilab.ops and nkilab.kernels.

Inputs may be NumPy arrays (float32 or ml_dtypes.bfloat16, the reference's types),
CPU tensors (pinned or pageable) or CUDA tensors; outputs come back in the container
type of the first input.
"""
from __future__ import annotations

import numpy as np
import torch


def bf16_numpy_dtype():
    import ml_dtypes

    return np.dtype(ml_dtypes.bfloat16)


def to_device(x, device=None) -> torch.Tensor:
    """NumPy / CPU tensor / CUDA tensor -> contiguous CUDA tensor (float32 or bfloat16)."""
    if isinstance(x, torch.Tensor):
        t = x
    else:
        a = np.asarray(x)
        if a.dtype == bf16_numpy_dtype():
            t = torch.from_numpy(np.ascontiguousarray(a).view(np.uint16)).view(torch.bfloat16)
        elif a.dtype == np.float32:
            t = torch.from_numpy(np.ascontiguousarray(a))
        else:
            raise TypeError(f"nkilab ops take float32 or bfloat16 arrays, got {a.dtype}")
    if t.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"nkilab ops take float32 or bfloat16 tensors, got {t.dtype}")
    if t.device.type != "cuda":
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        t = t.to(dev, non_blocking=t.is_pinned())
    return t.contiguous()


def like_input(out: torch.Tensor, ref):
    """Return `out` in the container type of the first input `ref`."""
    if isinstance(ref, torch.Tensor):
        if ref.device.type == "cuda":
            return out
        host = torch.empty(out.shape, dtype=out.dtype, pin_memory=ref.is_pinned())
        host.copy_(out)  # synchronous device -> host copy
        return host
    host = out.cpu()
    if host.dtype == torch.bfloat16:
        return host.view(torch.uint16).numpy().view(bf16_numpy_dtype())
    return host.numpy()


def dtype_of(x):
    return x.dtype if isinstance(x, torch.Tensor) else np.asarray(x).dtype

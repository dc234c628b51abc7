"""Minimal NumPy restatement of the NKI instructions the reference kernels call.

Used only by make_golden.py, in a container where the reference source tree is
present but the ``nki`` package (cp313 wheel from the Neuron index) is not. Installing
this module as ``nki`` / ``nki.isa`` / ``nki.language`` lets the reference's own kernel
source (nkilab/kernels/*.py) and host wrappers (nkilab/ops.py, nkilab/model.py) run
unmodified on the CPU, so their outputs can be stored as golden vectors.

Semantics restated from the public NKI ISA documentation:
  * every instruction computes in fp32 and rounds once to its destination tile's dtype
    (round-to-nearest-even for bfloat16, via ml_dtypes);
  * nc_matmul(dst, stationary, moving): dst (+)= stationary^T @ moving, fp32 accumulate;
  * activation(op, data, scale, bias): op(data * scale + bias); the optional free-axis
    reduction is taken over the fp32 results, before the destination rounding;
  * tensor_scalar / scalar_tensor_tensor: (data op0 operand0) op1 operand1, where an
    operand is a scalar or a per-partition [P, 1] column;
  * affine_select: keeps on_true where offset + channel_multiplier*p + sum(step*i) >= 0.
The transcendental functions are NumPy's fp32 ones; the hardware's are not pinned.
"""
from __future__ import annotations

import sys
import types

import numpy as np

F32 = np.float32


class HbmArray(np.ndarray):
    """ndarray with the two NKI tensor-view methods the reference kernels call."""

    def permute(self, axes):
        return np.transpose(self, axes).view(HbmArray)

    def broadcast(self, axis, n):
        shape = list(self.shape)
        shape[axis] = n
        return np.broadcast_to(self, shape).view(HbmArray)


def _f(x):
    if isinstance(x, np.ndarray):
        return np.asarray(x).astype(F32)
    return F32(x)


def _store(dst, val):
    dst[...] = np.asarray(val, dtype=F32).astype(dst.dtype)


_BIN = {
    "multiply": np.multiply, "add": np.add, "subtract": np.subtract, "divide": np.divide,
    "maximum": np.maximum, "minimum": np.minimum,
}


def _bin(op, a, b):
    return _BIN[op](_f(a), _f(b)).astype(F32)


def _act(op, x):
    if op == "exp":
        return np.exp(x)
    if op == "square":
        return x * x
    if op == "rsqrt":
        return (F32(1.0) / np.sqrt(x)).astype(F32)
    if op == "silu":
        return (x / (F32(1.0) + np.exp(-x))).astype(F32)
    raise NotImplementedError(op)


def _ndarray(shape, dtype, buffer=None):
    return np.zeros(shape, dtype=np.dtype(dtype)).view(HbmArray)


def dma_copy(dst, src, **_):
    _store(dst, _f(np.asarray(src)))


def nc_matmul(dst, stationary, moving, accumulate=False, **_):
    r = _f(np.asarray(stationary)).T @ _f(np.asarray(moving))
    if accumulate:
        r = _f(np.asarray(dst)) + r
    _store(dst, r)


def nc_transpose(dst, data, **_):
    _store(dst, _f(np.asarray(data)).T)


def tensor_copy(dst, src, engine=None, **_):
    _store(dst, _f(np.asarray(src)))


def tensor_scalar(dst, data, op0, operand0, op1=None, operand1=None, engine=None, **_):
    v = _bin(op0, np.asarray(data), operand0)
    if op1 is not None:
        v = _bin(op1, v, operand1)
    _store(dst, v)


def tensor_tensor(dst, data1, data2, op, **_):
    _store(dst, _bin(op, np.asarray(data1), np.asarray(data2)))


def scalar_tensor_tensor(dst, data, op0, operand0, op1, operand1, **_):
    _store(dst, _bin(op1, _bin(op0, np.asarray(data), operand0), np.asarray(operand1)))


def tensor_reduce(dst, op, data, axis, negate=False, **_):
    d = _f(np.asarray(data))
    r = d.max(axis=axis, keepdims=True) if op == "max" else d.sum(axis=axis, keepdims=True, dtype=F32)
    if negate:
        r = -r
    _store(dst, r)


def activation(dst, op, data, bias=None, scale=1.0, reduce_op=None, reduce_res=None, reduce_cmd=None, **_):
    x = _f(np.asarray(data)) * _f(scale)
    if bias is not None:
        x = (x + _f(np.asarray(bias))).astype(F32)
    y = _act(op, x.astype(F32)).astype(F32)
    _store(dst, y)
    if reduce_res is not None:
        _store(reduce_res, y.sum(axis=1, keepdims=True, dtype=F32))


def reciprocal(dst, data, **_):
    _store(dst, F32(1.0) / _f(np.asarray(data)))


def memset(dst, value, **_):
    _store(dst, np.full(dst.shape, value, dtype=F32))


def affine_select(dst, pattern, channel_multiplier, on_true_tile, on_false_value, cmp_op, offset, **_):
    src = _f(np.asarray(on_true_tile))
    p = np.arange(src.shape[0]).reshape(-1, 1)
    val = offset + channel_multiplier * p
    for step, num in pattern:
        val = val + step * np.arange(num).reshape(1, -1)
    assert cmp_op == "greater_equal"
    _store(dst, np.where(val >= 0, src, F32(on_false_value)))


def jit(fn=None, **_):
    return fn if fn is not None else (lambda f: f)


def simulate(kernel):
    def run(*args, **kwargs):
        args = [a.view(HbmArray) if isinstance(a, np.ndarray) else a for a in args]
        return np.asarray(kernel(*args, **kwargs)).view(np.ndarray)
    return run


def install() -> None:
    """Register this module as nki, nki.isa and nki.language."""
    nl = types.ModuleType("nki.language")
    nl.float32 = np.dtype(np.float32)
    nl.shared_hbm, nl.sbuf, nl.psum = "shared_hbm", "sbuf", "psum"
    nl.ndarray = _ndarray
    for name in ("multiply", "add", "subtract", "divide", "maximum", "minimum", "max", "exp", "square", "rsqrt",
                 "silu", "greater_equal"):
        setattr(nl, name, name)
    isa = types.ModuleType("nki.isa")
    for fn in (dma_copy, nc_matmul, nc_transpose, tensor_copy, tensor_scalar, tensor_tensor, scalar_tensor_tensor,
               tensor_reduce, activation, reciprocal, memset, affine_select):
        setattr(isa, fn.__name__, fn)
    isa.engine = types.SimpleNamespace(scalar="scalar", vector="vector", gpsimd="gpsimd")
    isa.reduce_cmd = types.SimpleNamespace(reset_reduce="reset_reduce")
    nki = types.ModuleType("nki")
    nki.jit = jit
    nki.simulate = simulate
    nki.isa = isa
    nki.language = nl
    sys.modules["nki"] = nki
    sys.modules["nki.isa"] = isa
    sys.modules["nki.language"] = nl

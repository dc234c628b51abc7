"""ctypes binding of the C ABI in include/nkilab.h (libnkilab_b200.so, built in-tree).

This is the only module that touches the shared library. It fails loudly: if the
library is missing, importing nkilab.ops raises instead of falling back to any other
implementation. Status codes become :class:`NklError` with the library's message.
"""
from __future__ import annotations

import ctypes
import os

LIB_NAME = "libnkilab_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

# dtype codes (nkl_dtype)
FLOAT32 = 0
BFLOAT16 = 1

# attention launch modes (NKL_ATTN_*)
ATTN_AUTO = 0
ATTN_ONE_TILE_UNSPLIT = 1
ATTN_TWO_TILE = 2
ATTN_TWO_GROUPS = 3

# status codes (nkl_status)
OK = 0
ERR_SHAPE = 1
ERR_DTYPE = 2
ERR_ALIGN = 3
ERR_CUDA = 4
ERR_ARG = 5
ERR_DEVICE = 7

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); one entry per function declared in include/nkilab.h
SIGNATURES = {
    "nkl_abi_version": (_int, []),
    "nkl_status_string": (ctypes.c_char_p, [_int]),
    "nkl_last_error": (ctypes.c_char_p, []),
    "nkl_check_device": (_int, [_p]),
    "nkl_set_sm_budget": (_int, [_int, _p]),
    "nkl_rmsnorm": (_int, [_p, _p, _p, _i64, _i64, _f, _int, _p]),
    "nkl_add_rmsnorm": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _f, _int, _p]),
    "nkl_softmax": (_int, [_p, _p, _i64, _i64, _int, _p]),
    "nkl_softmax_unfused_workspace_size": (_sz, [_i64, _i64]),
    "nkl_softmax_unfused": (_int, [_p, _p, _p, _sz, _i64, _i64, _int, _p]),
    "nkl_softmax_unfused_static": (_int, [_p, _p, _i64, _i64, _int, _p]),
    "nkl_swiglu": (_int, [_p, _p, _p, _i64, _i64, _int, _p]),
    "nkl_rope": (_int, [_p, _p, _i64, _i64, _i64, _f, _i64, _int, _p]),
    "nkl_matmul": (_int, [_p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "nkl_matmul_naive": (_int, [_p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "nkl_matmul_swiglu": (_int, [_p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "nkl_matmul_residual": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "nkl_matmul_f32out": (_int, [_p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "nkl_attention": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _f, _int, _p]),
    "nkl_attention_workspace_size": (_sz, [_i64, _i64, _i64, _int]),
    "nkl_attention_ws": (_int, [_p, _p, _p, _p, _p, _sz, _i64, _i64, _i64, _f, _int, _p]),
    "nkl_attention_strided": (_int, [_p, _p, _p, _p, _p, _sz, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                     _i64, _f, _int, _p]),
    "nkl_attention_gqa": (_int, [_p, _p, _p, _p, _p, _sz, _i64, _i64, _i64, _i64, _f, _int, _p]),
    "nkl_attention_mode_workspace_size": (_sz, [_i64, _i64, _i64, _int, _int]),
    "nkl_attention_mode": (_int, [_p, _p, _p, _p, _p, _sz, _i64, _i64, _i64, _f, _int, _int, _p]),
    "nkl_ipc_handle_bytes": (_sz, []),
    "nkl_ipc_alloc": (_int, [_sz, _p, _p]),
    "nkl_ipc_open": (_int, [_p, _p]),
    "nkl_ipc_close": (_int, [_p]),
    "nkl_ipc_free": (_int, [_p]),
    "nkl_attention_allgather": (_int, [_p, _p, _p, _p, _p, _int, _int, _i64, _i64, _p, _sz, _i64, _i64, _i64, _f, _int,
                                       _p]),
    "nkl_attention_naive_workspace_size": (_sz, [_i64, _i64, _int]),
    "nkl_attention_naive": (_int, [_p, _p, _p, _p, _p, _sz, _i64, _i64, _i64, _f, _int, _p]),
}

ABI_VERSION = 1
SOFTMAX_UNFUSED_STATIC_BYTES = 16 * 1024 * 1024  # NKL_SOFTMAX_UNFUSED_STATIC_BYTES


class NklError(RuntimeError):
    """A C-ABI call returned a non-zero nkl_status."""

    def __init__(self, func: str, status: int, message: str):
        self.func = func
        self.status = status
        super().__init__(f"{func} failed ({status}): {message}")


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_NAME} is not built at {LIB_PATH}; build it with "
            "`make -C nki-kernel-lab_b200` or `python -c 'import __graft_entry__ as g; g.build()'`")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.nkl_abi_version() != ABI_VERSION:
        raise ImportError(f"{LIB_NAME} ABI version {lib.nkl_abi_version()} != expected {ABI_VERSION}")
    return lib


lib = _load()


def check(func: str, status: int) -> None:
    if status != OK:
        msg = lib.nkl_last_error().decode(errors="replace")
        raise NklError(func, status, msg)


def call(func: str, *args) -> None:
    """Call a status-returning entry point and raise NklError on failure."""
    check(func, getattr(lib, func)(*args))


def check_device(stream: int | None = None) -> None:
    """Synchronise `stream` and raise if a kernel reported a device-side failure."""
    check("nkl_check_device", lib.nkl_check_device(stream))

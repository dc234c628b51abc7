"""The C-ABI library loads and exports every symbol include/nkilab.h declares, and
its host-side argument checks answer with the documented status codes (CPU only:
no call here reaches a kernel launch)."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "nkilab.h")


def declared_functions() -> dict[str, int]:
    """name -> number of parameters, for every function prototype in the header."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for m in re.finditer(r"\b(nkl_\w+)\s*\(([^)]*)\)\s*;", text):
        params = m.group(2).strip()
        out[m.group(1)] = 0 if params in ("", "void") else len(params.split(","))
    return out


@pytest.fixture(scope="module")
def native():
    from nkilab import _native

    return _native


def test_header_declares_the_op_set():
    names = set(declared_functions())
    for op in ("nkl_rmsnorm", "nkl_softmax", "nkl_softmax_unfused", "nkl_swiglu", "nkl_matmul", "nkl_matmul_naive",
               "nkl_attention", "nkl_attention_naive"):
        assert op in names


def test_library_exports_every_declared_symbol(native):
    raw = ctypes.CDLL(native.LIB_PATH)
    for name, nparams in declared_functions().items():
        assert hasattr(raw, name), f"{name} not exported"
        assert name in native.SIGNATURES, f"{name} has no ctypes signature"
        assert len(native.SIGNATURES[name][1]) == nparams, name


def test_version_and_status_strings(native):
    assert native.lib.nkl_abi_version() == native.ABI_VERSION
    assert native.lib.nkl_status_string(0) == b"ok"
    assert native.lib.nkl_status_string(1) == b"unsupported shape"
    assert native.lib.nkl_status_string(99) == b"unknown status"


FAKE = ctypes.c_void_p(4096)      # never dereferenced: every call below fails validation first
FAKE_ODD = ctypes.c_void_p(4104)  # 8-byte but not 16-byte aligned


def test_bad_dtype_and_shape_codes(native):
    L = native.lib
    assert L.nkl_rmsnorm(FAKE, FAKE, FAKE, 4, 8, 1e-6, 7, None) == native.ERR_DTYPE
    assert b"dtype" in L.nkl_last_error()
    assert L.nkl_rmsnorm(FAKE, FAKE, FAKE, 4, 0, 1e-6, native.FLOAT32, None) == native.ERR_SHAPE
    assert L.nkl_softmax(FAKE, FAKE, -1, 8, native.BFLOAT16, None) == native.ERR_SHAPE
    assert L.nkl_swiglu(None, FAKE, FAKE, 4, 8, native.FLOAT32, None) == native.ERR_ARG
    assert L.nkl_attention(FAKE, FAKE, FAKE, FAKE, 1, 128, 129, 0.1, native.FLOAT32, None) == native.ERR_SHAPE
    assert L.nkl_attention(FAKE, FAKE, FAKE, FAKE, 1, 128, 96, 0.1, native.BFLOAT16, None) == native.ERR_SHAPE
    assert L.nkl_matmul(FAKE, FAKE, FAKE, 16, 16, 7, native.BFLOAT16, None) == native.ERR_SHAPE
    assert L.nkl_matmul(FAKE_ODD, FAKE, FAKE, 16, 16, 16, native.BFLOAT16, None) == native.ERR_ALIGN


def test_empty_inputs_are_no_ops(native):
    L = native.lib
    assert L.nkl_rmsnorm(None, None, None, 0, 8, 1e-6, native.BFLOAT16, None) == native.OK
    assert L.nkl_softmax(None, None, 0, 8, native.FLOAT32, None) == native.OK
    assert L.nkl_swiglu(None, None, None, 0, 8, native.BFLOAT16, None) == native.OK
    assert L.nkl_matmul(None, None, None, 0, 8, 8, native.BFLOAT16, None) == native.OK
    assert L.nkl_attention(None, None, None, None, 0, 128, 64, 0.1, native.BFLOAT16, None) == native.OK
    assert L.nkl_attention(None, None, None, None, 2, 0, 64, 0.1, native.BFLOAT16, None) == native.OK


def test_workspace_sizes_and_checks(native):
    L = native.lib
    n = L.nkl_softmax_unfused_workspace_size(100, 1000)
    assert n >= 100 * 1000 * 4 + 2 * 100 * 4 and n % 256 == 0
    assert L.nkl_softmax_unfused_workspace_size(0, 10) == 0
    assert L.nkl_softmax_unfused(FAKE, FAKE, FAKE, n - 1, 100, 1000, native.FLOAT32, None) == native.ERR_ARG
    assert L.nkl_softmax_unfused(FAKE, FAKE, ctypes.c_void_p(4096 + 16), n, 100, 1000, native.FLOAT32,
                                 None) == native.ERR_ALIGN
    a = L.nkl_attention_naive_workspace_size(2, 300, native.BFLOAT16)
    assert a >= 2 * 300 * 300 * (4 + 2)
    assert L.nkl_attention_naive(FAKE, FAKE, FAKE, FAKE, FAKE, a - 1, 2, 300, 64, 0.125, native.BFLOAT16,
                                 None) == native.ERR_ARG


def test_errors_raise_with_message(native):
    with pytest.raises(native.NklError, match="nkl_matmul.*multiples of 8"):
        native.call("nkl_matmul", FAKE, FAKE, FAKE, 16, 16, 7, native.BFLOAT16, None)


def test_attention_strided_rejects_bad_strides_before_device_work(native):
    """Strides must be positive multiples of 8 elements and rows at least head_dim long;
    checked before any CUDA call."""
    L = native.lib
    ok = dict(qs=384, qh=128, ks=384, kh=128, os_=256, oh=128)
    def call(**kw):
        a = {**ok, **kw}
        return L.nkl_attention_strided(FAKE, FAKE, FAKE, FAKE, None, 0, 2, 2, 128, 128, a["qs"], a["qh"], a["ks"],
                                       a["kh"], a["os_"], a["oh"], 0.1, native.BFLOAT16, None)
    assert call(qs=388) == native.ERR_ALIGN
    assert call(kh=0) == native.ERR_ALIGN
    assert call(oh=-128) == native.ERR_ALIGN
    assert call(os_=64) == native.ERR_SHAPE


def test_sm_budget_is_per_thread_and_returns_the_previous_value(native):
    """nkl_set_sm_budget is host state only: it needs no GPU, it reports the value it
    replaces, rejects negative counts and is kept per host thread."""
    import threading

    L = native.lib
    prev = ctypes.c_int(-1)
    assert L.nkl_set_sm_budget(100, ctypes.byref(prev)) == native.OK and prev.value == 0
    seen = []

    def other():
        p = ctypes.c_int(-1)
        L.nkl_set_sm_budget(7, ctypes.byref(p))
        seen.append(p.value)

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen == [0]  # another thread starts from "all SMs"
    assert L.nkl_set_sm_budget(-1, None) == native.ERR_ARG
    assert L.nkl_set_sm_budget(0, ctypes.byref(prev)) == native.OK and prev.value == 100

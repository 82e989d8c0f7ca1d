"""The C ABI library builds, loads, exports every symbol include/reng_cuda.h
declares, and refuses bad arguments before touching a device (CPU only)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from conftest import ROOT


def declared_functions():
    with open(os.path.join(ROOT, "include", "reng_cuda.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(reng_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("reng_fp8_quantize", "reng_model_create", "reng_model_prefill",
                 "reng_model_decode", "reng_model_reset", "reng_model_destroy",
                 "reng_tp_unique_id", "reng_last_error"):
        assert must in names


def test_integration_ffi_stub_declares_every_function():
    """The Rust FFI stub a maintainer would add binds
    exactly the functions the header declares."""
    with open(os.path.join(ROOT, "INTEGRATION.md")) as f:
        stub = set(re.findall(r"pub fn (reng_[a-z0-9_]+)\(", f.read()))
    assert stub == set(declared_functions()), sorted(stub ^ set(declared_functions()))


def test_library_exports_every_declared_symbol(reng_lib):
    L = reng_lib.lib()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing
    # and the ctypes table covers them all
    assert set(declared_functions()) <= set(reng_lib.SIGNATURES)


def test_version_and_error_string(reng_lib):
    L = reng_lib.lib()
    assert L.reng_version() >= 1
    assert isinstance(L.reng_last_error(), bytes)


def test_quantize_refuses_bad_shapes_without_a_device(reng_lib):
    L = reng_lib.lib()
    w = np.zeros(4, np.uint16)
    codes = np.zeros(4, np.uint8)
    scales = np.zeros(1, np.float32)
    bias = C.c_uint32()
    p = lambda a: a.ctypes.data_as(C.c_void_p)
    rc = L.reng_fp8_quantize(p(w), 0, 4, 0, 0, 1.0, p(codes), p(scales), C.byref(bias), 1, None)
    assert rc == reng_lib.RENG_E_INVAL
    assert b"empty shape" in L.reng_last_error()
    rc = L.reng_fp8_quantize(p(w), 1, 4, 0, 0, 0.0, p(codes), p(scales), C.byref(bias), 1, None)
    assert rc == reng_lib.RENG_E_INVAL
    assert b"backoff" in L.reng_last_error()
    rc = L.reng_fp8_quantize(p(w), 1, 4, 7, 0, 1.0, p(codes), p(scales), C.byref(bias), 1, None)
    assert rc == reng_lib.RENG_E_INVAL
    with pytest.raises(reng_lib.RengError):
        reng_lib.check(rc)


def test_model_create_refuses_bad_descriptors_without_a_device(reng_lib):
    L = reng_lib.lib()
    out = C.c_void_p()
    d = reng_lib.ModelDesc()
    rc = L.reng_model_create(C.byref(d), None, None, None, None, None, None, 1, C.byref(out))
    assert rc == reng_lib.RENG_E_INVAL
    assert out.value is None

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


FFI_STUB = os.path.join(ROOT, "include", "reng_cuda_ffi.rs")


def test_integration_ffi_stub_declares_every_function():
    """The Rust FFI binding a maintainer adds to the reference
    (include/reng_cuda_ffi.rs) binds exactly the functions the header
    declares."""
    with open(FFI_STUB) as f:
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
    assert L.reng_version() == 3   # the struct layouts and entry points of this header
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
    # the allocation-free entry runs the same checks and names itself
    rc = L.reng_fp8_quantize_noalloc(p(w), 0, 4, 0, 0, 1.0, p(codes), p(scales), C.byref(bias), None)
    assert rc == reng_lib.RENG_E_INVAL
    assert L.reng_last_error().startswith(b"reng_fp8_quantize_noalloc: empty shape")


def test_model_create_refuses_bad_descriptors_without_a_device(reng_lib):
    L = reng_lib.lib()
    out = C.c_void_p()
    d = reng_lib.ModelDesc()
    rc = L.reng_model_create(C.byref(d), None, None, None, None, None, None, 1, C.byref(out))
    assert rc == reng_lib.RENG_E_INVAL
    assert out.value is None


def test_ctypes_structs_match_the_header_layout(tmp_path):
    """Size and field offsets of every struct the header declares, as gcc
    lays them out, against the ctypes mirrors the Python host passes."""
    import ctypes as C
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("no gcc")
    from reng import _lib
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    structs = {"reng_model_desc": _lib.ModelDesc, "reng_layer_weights": _lib.LayerWeights,
               "reng_step_times": _lib.StepTimes, "reng_device_info": _lib.DeviceInfo}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "reng_cuda.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append('printf("%s size %%zu\\n", sizeof(%s));' % (cname, cname))
        for fname, _ in py._fields_:
            lines.append('printf("%s %s %%zu\\n", offsetof(%s, %s));' % (cname, fname, cname, fname))
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(root, "include"), str(src), "-o", str(exe)],
                   check=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        a, b, v = line.split()
        got[(a, b)] = int(v)
    for cname, py in structs.items():
        assert got[(cname, "size")] == C.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)


@pytest.mark.gpu
def test_device_discovery_agrees_with_torch(reng_lib):
    import torch
    from reng._lib import devices
    d = devices()
    assert len(d) == torch.cuda.device_count() >= 1
    for i, rec in enumerate(d):
        p = torch.cuda.get_device_properties(i)
        assert rec["ordinal"] == i and rec["name"] and ":" in rec["pci_bus_id"]
        assert rec["sm_count"] == p.multi_processor_count
        assert rec["compute_capability"] == (p.major, p.minor)
        assert rec["total_bytes"] == p.total_memory


def test_bindings_refuse_a_library_of_another_abi_version(monkeypatch):
    """A library built from another header would be handed structs of the
    wrong size: the bindings stop at load time instead."""
    from reng import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "ABI_VERSION", _lib.ABI_VERSION + 1)
    with pytest.raises(OSError, match="ABI version"):
        _lib.lib()
    monkeypatch.undo()
    assert _lib.lib().reng_version() == _lib.ABI_VERSION


def _header_struct_fields(text, name):
    """Field names, in order, of `typedef struct name { ... } name;` in C."""
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), text, re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    names = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        for part in decl.split(","):
            part = re.sub(r"\[.*?\]", "", part).strip()
            names.append(re.findall(r"[A-Za-z_][A-Za-z0-9_]*", part)[-1])
    return names


def _stub_struct_fields(text, name):
    body = re.search(r"pub struct %s \{(.*?)\}" % name, text, re.S).group(1)
    return re.findall(r"pub ([a-z_0-9]+):", body)


def test_integration_ffi_stub_structs_match_the_header():
    """Every struct of the header appears in the Rust stub with the same
    fields in the same order (the layout a #[repr(C)] mirror needs)."""
    with open(os.path.join(ROOT, "include", "reng_cuda.h")) as f:
        header = f.read()
    with open(FFI_STUB) as f:
        stub = f.read()
    structs = re.findall(r"typedef struct (reng_[a-z_]+) \{", header)
    assert {"reng_model_desc", "reng_layer_weights", "reng_step_times", "reng_device_info"} <= set(structs)
    for name in structs:
        assert _stub_struct_fields(stub, name) == _header_struct_fields(header, name), name

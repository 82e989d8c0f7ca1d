"""The allocation-free FP8 quantizer entry point (reng_fp8_quantize_noalloc).

Some callers cannot allocate device memory: a process whose GPU memory is
already reserved by another framework's allocator, or a code path that must
not enter the CUDA allocator at all.  For them the library stages the matrix
in a fixed device array instead of memory allocated per call.  These tests
call that entry point through the C ABI and require its codes, scales and
exponent bias to equal those of the allocating entry point
(reng_fp8_quantize with host buffers) bit for bit -- the quantizer's parity
bar -- on two calls in a row, so that contents the first call leaves in the
shared array cannot leak into the second.  The file sorts last so that a run
stopped at a first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _quantize(lib, fn, w, rows, cols, fmt, scaling, backoff=1.0):
    codes = np.empty(rows * cols, np.uint8)
    scales = np.empty(rows, np.float32)
    bias = C.c_uint32(0)
    args = [w.ctypes.data, rows, cols, fmt, scaling, backoff, codes.ctypes.data, scales.ctypes.data,
            C.byref(bias)]
    if fn == "reng_fp8_quantize":
        args.append(lib.RENG_MEM_HOST)
    args.append(None)
    lib.call(fn, *args)
    return codes, scales, bias.value


def test_noalloc_quantize_matches_the_allocating_entry_point(reng_lib):
    import torch
    torch.cuda.init()
    from reng.synth import f32_to_bf16_bits, fp8_config0_matrix
    lib = reng_lib
    # two different calls in a row: the second must not see the first's leftovers
    cases = [
        (fp8_config0_matrix(1024, 2048, seed=11), 1024, 2048, 0, 1),   # E4M3, hw exponent bias
        (fp8_config0_matrix(512, 1000, seed=12), 512, 1000, 1, 0),     # E5M2, per channel, ragged cols
    ]
    x = np.random.default_rng(3).standard_normal(96 * 64).astype(np.float32)
    x[:5] = [np.inf, -np.inf, np.nan, 0.0, 1e-40]
    cases.append((f32_to_bf16_bits(x), 96, 64, 0, 0))                  # specials, per channel
    for w, rows, cols, fmt, scaling in cases:
        want = _quantize(lib, "reng_fp8_quantize", w, rows, cols, fmt, scaling)
        for _ in range(2):
            got = _quantize(lib, "reng_fp8_quantize_noalloc", w, rows, cols, fmt, scaling)
            assert got[2] == want[2]
            assert np.array_equal(got[1].view(np.uint32), want[1].view(np.uint32))
            assert np.array_equal(got[0], want[0])


def test_noalloc_quantize_refuses_matrices_beyond_its_scratch(reng_lib):
    lib = reng_lib
    w = np.zeros(1, np.uint16)  # never read: the size check comes first
    out = np.zeros(1, np.uint8)
    sc = np.zeros(1, np.float32)
    bias = C.c_uint32(0)
    for rows, cols in ((65537, 1), (2048, 2048)):
        rc = lib.lib().reng_fp8_quantize_noalloc(w.ctypes.data, rows, cols, 0, 0, 1.0, out.ctypes.data,
                                                 sc.ctypes.data, C.byref(bias), None)
        assert rc == lib.RENG_E_INVAL
        assert b"exceeds the fixed scratch" in lib.lib().reng_last_error()

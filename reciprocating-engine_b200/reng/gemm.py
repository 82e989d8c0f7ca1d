"""The packed tcgen05 GEMM on its own: y = x @ w.T in f32 from bf16 bit
patterns (the projection kernel of steps with more than 8 rows).

    y, ms = gemm_bf16(w_bits, x_bits, splits=0, iters=0)

w_bits: uint16 [rows][K] bf16 bits, x_bits: uint16 [M][K] (1 <= M <= 1024,
N-tiles of 256 rows beyond 256; K % 8 == 0).  iters > 0 also times the kernel alone (mean ms per launch).
"""
import ctypes as C

import numpy as np

from . import _lib


def gemm_bf16(w_bits, x_bits, splits=0, iters=0):
    w = np.ascontiguousarray(w_bits, dtype=np.uint16)
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    if w.ndim != 2 or x.ndim != 2 or w.shape[1] != x.shape[1]:
        raise ValueError("w [rows][K] and x [M][K] must share K")
    rows, K = w.shape
    M = x.shape[0]
    y = np.empty((M, rows), np.float32)
    ms = C.c_float(0.0)
    _lib.call("reng_gemm_bf16", w.ctypes.data, rows, K, x.ctypes.data, M, y.ctypes.data, splits, iters,
              C.byref(ms), _lib.RENG_MEM_HOST)
    return y, float(ms.value)

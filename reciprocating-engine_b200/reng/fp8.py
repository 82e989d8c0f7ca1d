"""The reference's `reng-fp8` quantize API over the CUDA quantizer.

Mirrors crates/reng-fp8/src/lib.rs: `Fp8Format` (lib.rs:53-147),
`Scaling` (lib.rs:240-275), `Quantized` (lib.rs:291-345),
`quantize` / `quantize_with` (lib.rs:492-563) and `DEFAULT_BACKOFF`
(lib.rs:484).  The arithmetic runs on the GPU (libreng_cuda.so,
reng_fp8_quantize); the results are bit-identical to the reference's host
quantizer.  Shape misuse raises ValueError where the reference panics.
"""
import ctypes as C
import enum
from dataclasses import dataclass

import numpy as np

from . import _lib

DEFAULT_BACKOFF = 1.0


class Fp8Format(enum.IntEnum):
    E4M3 = _lib.RENG_FP8_E4M3
    E5M2 = _lib.RENG_FP8_E5M2

    @property
    def mantissa_bits(self):
        return 3 if self is Fp8Format.E4M3 else 2

    @property
    def exponent_bits(self):
        return 7 - self.mantissa_bits

    @property
    def exponent_bias(self):
        return 7 if self is Fp8Format.E4M3 else 15

    @property
    def max_finite_code(self):
        m = self.mantissa_bits
        return (((1 << self.exponent_bits) - 2) << m) | ((1 << m) - 1)

    @property
    def max_finite(self):
        return 240.0 if self is Fp8Format.E4M3 else 57344.0

    @property
    def hw_exponent_biases(self):
        return (15, 11, 7, 3) if self is Fp8Format.E4M3 else (15,)

    @property
    def short_name(self):
        return "e4m3" if self is Fp8Format.E4M3 else "e5m2"

    @staticmethod
    def from_name(s):
        s = s.strip().lower()
        if s in ("e4m3", "fp8_143", "hf8"):
            return Fp8Format.E4M3
        if s in ("e5m2", "fp8_152", "f8"):
            return Fp8Format.E5M2
        return None


class Scaling(enum.IntEnum):
    PerChannel = _lib.RENG_SCALING_PCS
    HwExpBias = _lib.RENG_SCALING_HW
    Unit = _lib.RENG_SCALING_UNIT

    @staticmethod
    def from_name(s):
        s = s.strip().lower()
        if s in ("pcs", "per-channel", "perchannel"):
            return Scaling.PerChannel
        if s in ("hw", "hw-exp-bias", "expbias"):
            return Scaling.HwExpBias
        if s in ("unit", "none"):
            return Scaling.Unit
        return None

    @property
    def short_name(self):
        return {0: "pcs", 1: "hw", 2: "unit"}[int(self)]


@dataclass
class Quantized:
    format: Fp8Format
    scaling: Scaling
    rows: int
    cols: int
    codes: np.ndarray   # u8 [rows * cols]
    scales: np.ndarray  # f32 [rows]
    exp_bias: int

    def code_bytes(self):
        return self.codes.size

    def scale_operand(self):
        return self.scales if self.scaling == Scaling.PerChannel else None


def _check(w_size, rows, cols, backoff):
    if rows <= 0 or cols <= 0:
        raise ValueError("empty shape %d x %d" % (rows, cols))
    if w_size != rows * cols:
        raise ValueError("weight length %d against the shape %d x %d" % (w_size, rows, cols))
    if not (backoff > 0.0 and np.isfinite(backoff)):
        raise ValueError("backoff %r is not positive and finite" % (backoff,))


def quantize_with(w, rows, cols, fmt, scaling, backoff):
    """Quantize host bf16 bits `w` ([rows*cols] u16) on the GPU; returns Quantized."""
    w = np.ascontiguousarray(w, dtype=np.uint16).reshape(-1)
    _check(w.size, rows, cols, backoff)
    codes = np.empty(rows * cols, np.uint8)
    scales = np.empty(rows, np.float32)
    bias = C.c_uint32(0)
    _lib.call("reng_fp8_quantize", w.ctypes.data, rows, cols, int(fmt), int(scaling),
              float(backoff), codes.ctypes.data, scales.ctypes.data, C.byref(bias),
              _lib.RENG_MEM_HOST, None)
    return Quantized(Fp8Format(fmt), Scaling(scaling), rows, cols, codes, scales, int(bias.value))


def quantize(w, rows, cols, fmt, scaling):
    return quantize_with(w, rows, cols, fmt, scaling, DEFAULT_BACKOFF)


def quantize_device(w, rows, cols, fmt, scaling, backoff=DEFAULT_BACKOFF, codes=None,
                    scales=None, stream=None):
    """Quantize a device tensor (torch, bf16 or int16 bits) in HBM.

    Returns (codes uint8 [rows, cols], scales f32 [rows], exp_bias)."""
    import torch
    if w.numel() != rows * cols:
        raise ValueError("weight length against the shape")
    _check(w.numel(), rows, cols, backoff)
    dev = w.device
    if codes is None:
        codes = torch.empty((rows, cols), dtype=torch.uint8, device=dev)
    if scales is None:
        scales = torch.empty(rows, dtype=torch.float32, device=dev)
    bias = C.c_uint32(0)
    st = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
    _lib.call("reng_fp8_quantize", w.data_ptr(), rows, cols, int(fmt), int(scaling),
              float(backoff), codes.data_ptr(), scales.data_ptr(), C.byref(bias),
              _lib.RENG_MEM_DEVICE, st)
    return codes, scales, int(bias.value)

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

    def dequantize(self):
        """The matrix back in f32, [rows * cols] row-major: decode(code) *
        scale, one f32 multiply per element (lib.rs:316-327)."""
        codes = np.asarray(self.codes, np.uint8).reshape(self.rows, self.cols)
        vals = decode_table(self.format)[codes]
        return (vals * np.asarray(self.scales, np.float32)[:, None]).astype(np.float32).reshape(-1)

    def dequantize_bf16(self):
        """bf16 bits of dequantize(), one rounding per element (lib.rs:331-335)."""
        from .synth import f32_to_bf16_bits
        return f32_to_bf16_bits(self.dequantize())


def _pow2(e):
    """2^e as an exact f32 for e in -149..127 (lib.rs:229-236)."""
    return np.float32(np.ldexp(np.float32(1.0), int(e)))


_DECODE = {}


def decode_table(fmt):
    """f32 value of every code (decode, lib.rs:205-225): the finite values
    exactly, the reserved top exponent field as an infinity (zero mantissa)
    or a NaN."""
    fmt = Fp8Format(fmt)
    if fmt not in _DECODE:
        mb, bias, eb = fmt.mantissa_bits, fmt.exponent_bias, fmt.exponent_bits
        out = np.empty(256, np.float32)
        for code in range(256):
            sign = np.float32(-1.0 if code & 0x80 else 1.0)
            mant = code & ((1 << mb) - 1)
            ef = (code & 0x7F) >> mb
            if ef == (1 << eb) - 1:
                out[code] = sign * np.float32(np.inf) if mant == 0 else np.float32(np.nan)
                continue
            frac = np.float32(mant) / np.float32(1 << mb)
            if ef == 0:
                out[code] = sign * frac * _pow2(1 - bias)
            else:
                out[code] = sign * (np.float32(1.0) + frac) * _pow2(ef - bias)
        out.setflags(write=False)
        _DECODE[fmt] = out
    return _DECODE[fmt]


def decode(code, fmt):
    """One code to f32 (lib.rs:205-225)."""
    return float(decode_table(fmt)[int(code) & 0xFF])


@dataclass
class RowError:
    """Mean and maximum of |w - dequant(w)| / |w| over one row's non-zero
    weights (lib.rs:339-345)."""
    mean_rel: float
    max_rel: float


def _row_error(w_row, codes_row, scale, fmt):
    from .synth import bf16_bits_to_f32
    want = bf16_bits_to_f32(np.asarray(w_row, np.uint16))
    nz = want != 0.0
    if not nz.any():
        return RowError(0.0, 0.0)
    got = decode_table(fmt)[np.asarray(codes_row, np.uint8)[nz]] * np.float32(scale)
    rel = np.abs((got - want[nz]) / want[nz]).astype(np.float32)
    # the reference sums in order in f64: a running sum, not a pairwise one
    total = np.cumsum(rel.astype(np.float64))[-1]
    # the scan's f32::max starts at 0 and never takes a NaN
    seen = rel[~np.isnan(rel)]
    mx = seen.max() if seen.size else np.float32(0.0)
    return RowError(float(np.float32(total / rel.size)), float(np.float32(mx)))


def row_errors(w, q):
    """Per-row relative error of `q` against the bf16 bits `w` it came from
    (row_errors, lib.rs:347-386); an all-zero row reports 0.0 for both."""
    w = np.asarray(w, np.uint16).reshape(-1)
    if w.size != q.rows * q.cols:
        raise ValueError("the weights hold %d values, not rows x cols" % w.size)
    codes = np.asarray(q.codes, np.uint8).reshape(q.rows, q.cols)
    w = w.reshape(q.rows, q.cols)
    return [_row_error(w[r], codes[r], q.scales[r], q.format) for r in range(q.rows)]


def sample_row_errors(w, q, max_rows):
    """row_errors over at most `max_rows` evenly spaced rows, every
    ceil(rows / n)-th from row 0 (sample_row_errors, lib.rs:388-430)."""
    w = np.asarray(w, np.uint16).reshape(-1)
    if w.size != q.rows * q.cols:
        raise ValueError("the weights hold %d values, not rows x cols" % w.size)
    if max_rows <= 0:
        raise ValueError("max_rows must be positive")
    n = min(max_rows, q.rows)
    step = -(-q.rows // n)
    codes = np.asarray(q.codes, np.uint8).reshape(q.rows, q.cols)
    w = w.reshape(q.rows, q.cols)
    return [_row_error(w[r], codes[r], q.scales[r], q.format) for r in range(0, q.rows, step)]


def row_absmax(w, rows, cols):
    """Largest magnitude of each row of bf16 bits [rows, cols], NaN never
    chosen (row_absmax, lib.rs:432-455)."""
    from .synth import bf16_bits_to_f32
    w = np.asarray(w, np.uint16).reshape(-1)
    if w.size != rows * cols:
        raise ValueError("the weights hold %d values, not rows x cols" % w.size)
    a = np.abs(bf16_bits_to_f32(w).reshape(rows, cols))
    a = np.where(np.isnan(a), np.float32(0.0), a)
    return a.max(axis=1).astype(np.float32)


def choose_exp_bias(absmax, fmt):
    """The largest hardware exponent bias whose range max_finite *
    2^(default - b) still covers `absmax`; the widest bias otherwise
    (choose_exp_bias, lib.rs:457-475)."""
    fmt = Fp8Format(fmt)
    a = np.float32(absmax)
    for b in fmt.hw_exponent_biases:
        if a <= np.float32(fmt.max_finite) * _pow2(fmt.exponent_bias - b):
            return b
    return fmt.hw_exponent_biases[-1]


def _check(w_size, rows, cols, backoff):
    if rows <= 0 or cols <= 0:
        raise ValueError("empty shape %d x %d" % (rows, cols))
    if w_size != rows * cols:
        raise ValueError("the weights hold %d values, not %d x %d" % (w_size, rows, cols))
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
        raise ValueError("the weights hold %d values, not rows x cols" % w.numel())
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


# Rows per matrix the model-level pass measures its error on (FP8_ERROR_ROWS,
# crates/reng-model/src/lib.rs:1853).
FP8_ERROR_ROWS = 8
PROJECTIONS = ("wq", "wk", "wv", "wo", "wg", "wu", "wd")


@dataclass
class Fp8Report:
    """What one model quantization pass produced (Fp8Report,
    crates/reng-model/src/lib.rs:1827-1876)."""
    matrices: int = 0
    bf16_bytes: int = 0
    fp8_bytes: int = 0
    scale_bytes: int = 0
    mean_rel: float = 0.0
    max_rel: float = 0.0
    secs: float = 0.0

    def __str__(self):
        gib = 1024.0 ** 3
        return ("%d matrices, %.2f GiB bf16 -> %.2f GiB fp8 + %d KiB scales, mean rel %.4f, "
                "max rel %.4f, %.2f s" % (self.matrices, self.bf16_bytes / gib, self.fp8_bytes / gib,
                                           self.scale_bytes // 1024, self.mean_rel, self.max_rel,
                                           self.secs))


def quantize_model(w, cfg, fmt=Fp8Format.E4M3, scaling=Scaling.PerChannel, backoff=DEFAULT_BACKOFF,
                   quantizer=None):
    """The seven projections of every layer quantized, norms / embedding /
    LM head left bf16 (LlamaWeights::quantize_fp8, lib.rs:1878-1937).
    Returns (layers, report): layers[l] maps "wq".."wd" to Quantized, and the
    report samples FP8_ERROR_ROWS rows per matrix.  `quantizer(w, rows,
    cols, fmt, scaling, backoff) -> Quantized` defaults to quantize_with
    (the GPU quantizer).  The engine's own FP8 path quantizes on the device
    at create time with the same rules; this is the host API around it."""
    import time
    q = quantizer or quantize_with
    t0 = time.perf_counter()
    h, inter, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim()
    qd, kvd = cfg.q_dim(), cfg.n_kv_heads() * hd
    shapes = {"wq": (qd, h), "wk": (kvd, h), "wv": (kvd, h), "wo": (h, qd), "wg": (inter, h),
              "wu": (inter, h), "wd": (h, inter)}
    rep, errors, out = Fp8Report(), [], []
    for li, lw in enumerate(w["layers"]):
        layer = {}
        for name in PROJECTIONS:
            rows, cols = shapes[name]
            m = np.asarray(lw[name], np.uint16).reshape(-1)
            if m.size != rows * cols:
                raise ValueError("layer %d %s: %d elements, expected %d x %d"
                                 % (li, name, m.size, rows, cols))
            qm = q(m, rows, cols, fmt, scaling, backoff)
            rep.matrices += 1
            rep.bf16_bytes += m.size * 2
            rep.fp8_bytes += qm.code_bytes()
            rep.scale_bytes += len(qm.scales) * 4
            errors += sample_row_errors(m, qm, FP8_ERROR_ROWS)
            layer[name] = qm
        out.append(layer)
    if errors:
        rep.mean_rel = float(np.float32(np.cumsum(np.array([e.mean_rel for e in errors],
                                                            np.float64))[-1] / len(errors)))
        rep.max_rel = float(max(0.0, max((e.max_rel for e in errors
                                          if not np.isnan(e.max_rel)), default=0.0)))
    rep.secs = time.perf_counter() - t0
    return out, rep

"""Seeded synthetic inputs of the benchmark configurations.

No checkpoints or datasets are available, so every workload is synthetic:
weight matrices drawn N(0, 0.02) with numpy's default_rng, rounded to bf16
(round to nearest even), and prompts of uniform-random token ids.
"""
import numpy as np


def f32_to_bf16_bits(x):
    """Round f32 to bf16 bits (RNE, NaN -> 0x7fc0), the reference's conversion."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7fffffff) > 0x7f800000
    r = ((u + (0x7fff + ((u >> 16) & 1))) >> 16).astype(np.uint16)
    r[nan] = 0x7fc0
    return r


def bf16_bits_to_f32(b):
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def fp8_config0_matrix(rows=4096, cols=4096, seed=0, outlier_frac=0.001, outlier_scale=50.0):
    """The quantizer workload: bf16 [rows, cols], N(0, 0.02), with a fixed-seed
    `outlier_frac` of the entries scaled x50 so saturation paths are exercised."""
    rng = np.random.default_rng(seed)
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    n_out = int(round(rows * cols * outlier_frac))
    idx = rng.choice(rows * cols, size=n_out, replace=False)
    w[idx] *= np.float32(outlier_scale)
    return f32_to_bf16_bits(w)


def prompt_ids(n, vocab, seed=0):
    """A uniform-random prompt of n token ids."""
    return np.random.default_rng(seed).integers(0, vocab, size=n, dtype=np.int64).astype(np.uint32)

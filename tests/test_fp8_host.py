"""The host report side of the reng-fp8 API (reng/fp8.py): decode,
Quantized.dequantize / dequantize_bf16, row_errors, sample_row_errors,
row_absmax and choose_exp_bias, as crates/reng-fp8/src/lib.rs:205-475 define
them.  The codes and scales come from the C restatement of the quantizer,
so this runs on CPU; every result must equal the restatement's bit for bit,
and the sampling test is the reference's own (lib.rs:884-900)."""
import numpy as np
import pytest


def bits(x):
    from reng.synth import f32_to_bf16_bits
    return f32_to_bf16_bits(np.asarray(x, np.float32))


def quantized(w, rows, cols, fmt, scaling):
    import oracle
    from reng.fp8 import Fp8Format, Quantized, Scaling
    codes, scales, bias = oracle.quantize(w, rows, cols, int(fmt), int(scaling))
    return Quantized(Fp8Format(fmt), Scaling(scaling), rows, cols, codes, scales, bias)


def weights(rows, cols, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    w[rng.random((rows, cols)) < 0.01] *= 50.0
    w[0, :5] = 0.0
    w[2] = 0.0                       # an all-zero row
    w[3, 7] = 1e-30                  # a quotient in the fp8 subnormal range
    return bits(w)


@pytest.mark.parametrize("fmt", [0, 1])
def test_decode_table_matches_the_restatement(oracle_lib, fmt):
    import oracle
    from reng.fp8 import Fp8Format, decode, decode_table
    f = Fp8Format(list(Fp8Format)[fmt])
    t = decode_table(f)
    for c in range(256):
        want = oracle.decode(c, int(f))
        got = t[c]
        assert (np.isnan(want) and np.isnan(got)) or np.float32(want).tobytes() == got.tobytes(), c
    assert decode(0x3B, Fp8Format.E4M3) == 1.375 and decode(0x77, Fp8Format.E4M3) == 240.0


@pytest.mark.parametrize("fmt,scaling", [(0, 0), (1, 0), (0, 1), (0, 2)])
def test_dequantize_and_row_errors_equal_the_restatement(oracle_lib, fmt, scaling):
    import oracle
    from reng.fp8 import Fp8Format, Scaling, row_errors
    f, s = list(Fp8Format)[fmt], list(Scaling)[scaling]
    rows, cols = 24, 200
    w = weights(rows, cols, 10 + fmt + 3 * scaling)
    q = quantized(w, rows, cols, f, s)
    want = oracle.dequantize(q.codes, q.scales, rows, cols, int(f))
    assert q.dequantize().tobytes() == want.tobytes()
    from reng.synth import f32_to_bf16_bits
    assert np.array_equal(q.dequantize_bf16(), f32_to_bf16_bits(want))
    mean, mx = oracle.row_errors(w, q.codes, q.scales, rows, cols, int(f))
    errs = row_errors(w, q)
    assert np.array([e.mean_rel for e in errs], np.float32).tobytes() == mean.tobytes()
    assert np.array([e.max_rel for e in errs], np.float32).tobytes() == mx.tobytes()
    assert errs[2].mean_rel == 0.0 and errs[2].max_rel == 0.0


def test_sampling_agrees_with_the_full_error_pass(oracle_lib):
    """lib.rs:884-900, with the reference's own weights."""
    from reng.fp8 import Fp8Format, Scaling, row_errors, sample_row_errors
    rows, cols = 16, 64
    w = bits([(((i * 37) % 101) - 50.0) / 50.0 for i in range(rows * cols)])
    q = quantized(w, rows, cols, Fp8Format.E4M3, Scaling.PerChannel)
    full = row_errors(w, q)
    assert sample_row_errors(w, q, rows) == full
    s = sample_row_errors(w, q, 4)
    assert len(s) == 4 and all(e == full[4 * k] for k, e in enumerate(s))
    assert len(sample_row_errors(w, q, 1000)) == rows
    with pytest.raises(ValueError):
        sample_row_errors(w, q, 0)


def test_row_absmax_and_exp_bias_choice_equal_the_restatement(oracle_lib):
    import oracle
    from reng.fp8 import Fp8Format, choose_exp_bias, row_absmax
    rows, cols = 8, 96
    w = weights(rows, cols, 3).copy()
    w[4, 9] = 0x7FC0                 # a NaN weight is never the maximum
    w[5, 1] = 0xFF80                 # -inf is
    got = row_absmax(w, rows, cols)
    want = np.empty(rows, np.float32)
    lib = oracle.lib()
    lib.orc_row_absmax(oracle._p(np.ascontiguousarray(w)), rows, cols, oracle._p(want))
    assert got.tobytes() == want.tobytes()
    for fmt in Fp8Format:
        for a in (0.0, 0.5, 0.9375, 0.94, 15.0, 15.5, 240.0, 241.0, 3840.0, 5000.0, 57344.0, 1e6):
            assert choose_exp_bias(a, fmt) == lib.orc_choose_exp_bias(a, int(fmt)), (fmt, a)
    assert choose_exp_bias(15.0, Fp8Format.E4M3) == 11 and choose_exp_bias(5000.0, Fp8Format.E4M3) == 3


def test_model_quantization_pass_and_report(oracle_lib):
    """quantize_model over a small Llama: seven matrices per layer, byte
    counts, the sampled error summary, and the reference's report line
    (lib.rs:1827-1937).  The quantizer is the C restatement here (CPU)."""
    import oracle
    from reng.config import LlamaConfig
    from reng.fp8 import Fp8Format, Quantized, Scaling, quantize_model, row_errors
    from reng.weights import random_weights
    cfg = LlamaConfig(hidden_size=64, intermediate_size=96, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim_=16, vocab_size=50,
                      model_type="llama")
    w = random_weights(cfg, seed=4)

    def host_quantizer(m, rows, cols, fmt, scaling, backoff):
        c, s, b = oracle.quantize(m, rows, cols, int(fmt), int(scaling), backoff)
        return Quantized(Fp8Format(fmt), Scaling(scaling), rows, cols, c, s, b)

    layers, rep = quantize_model(w, cfg, quantizer=host_quantizer)
    assert len(layers) == 2 and sorted(layers[0]) == sorted(("wq", "wk", "wv", "wo", "wg", "wu", "wd"))
    per_layer = 64 * 64 * 2 + 32 * 64 * 2 + 96 * 64 * 3
    assert rep.matrices == 14 and rep.fp8_bytes == 2 * per_layer and rep.bf16_bytes == 4 * per_layer
    assert rep.scale_bytes == 4 * 2 * (64 + 32 + 32 + 64 + 96 + 96 + 64)
    full = row_errors(w["layers"][1]["wd"], layers[1]["wd"])
    assert rep.max_rel >= max(e.max_rel for e in full[::8])
    assert 0.0 < rep.mean_rel < 0.05 and rep.max_rel < 0.07
    line = str(rep)
    assert line.startswith("14 matrices, 0.00 GiB bf16 -> 0.00 GiB fp8 + ") and "mean rel" in line
    with pytest.raises(ValueError):
        bad = {"layers": [dict(w["layers"][0], wq=w["layers"][0]["wq"][:10])]}
        quantize_model(bad, cfg, quantizer=host_quantizer)

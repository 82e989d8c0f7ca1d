"""The CPU oracle of the FP8 quantizer, pinned to the reference's own answers.

Mirrors the reference's tests: the unit known answers of
crates/reng-fp8/src/lib.rs:632-926 and the golden-file assertions of
crates/reng-fp8/tests/fixtures.rs:113-292 (fixture: tests/golden/fp8_cast.json).
"""
import json
import math
import os

import numpy as np
import pytest

from conftest import GOLDEN

E4M3, E5M2 = 0, 1
PCS, HW, UNIT = 0, 1, 2
FMT = {"e4m3": E4M3, "e5m2": E5M2}
SCL = {"pcs": PCS, "hw": HW, "unit": UNIT}


def bf(o, xs):
    return np.array([o.f32_to_bf16(x) for x in xs], np.uint16)


def load_cases():
    with open(os.path.join(GOLDEN, "fp8_cast.json")) as f:
        doc = json.load(f)
    out = []
    for c in doc["cases"]:
        if c["bf16_from"]:
            w = next(o for o in out if o["name"] == c["bf16_from"])["w"]
        else:
            h = c["bf16_hex"]
            w = np.array([int(h[i:i + 4], 16) for i in range(0, len(h), 4)], np.uint16)
        d = dict(c)
        d["w"] = w
        d["codes"] = np.frombuffer(bytes.fromhex(c["codes_hex"]), np.uint8)
        if c.get("torch_raw_hex"):
            d["torch_raw"] = np.frombuffer(bytes.fromhex(c["torch_raw_hex"]), np.uint8)
        d["scales"] = np.array(c["scale_bits"], np.uint32)
        out.append(d)
    return doc, out


# ----------------------------------------------------------- known answers --

def test_e4m3_codes_match_the_device_cast(oracle_lib):
    o = oracle_lib
    cases = [(0.0, 0x00), (1.0, 0x38), (1.375, 0x3b), (-3.3, 0xc5), (100.0, 0x6c),
             (0.01, 0x05), (0.0625, 0x18), (17.0, 0x58), (240.0, 0x77), (-240.0, 0xf7),
             (250.0, 0x77), (300.0, 0x77), (0.001, 0x01), (1e-9, 0x00),
             (math.inf, 0x77), (-math.inf, 0xf7)]
    for x, code in cases:
        assert o.encode(x, E4M3) == code, x
    assert o.encode(math.nan, E4M3) & 0x7f == 0x7f


def test_e5m2_codes_match_the_device_cast(oracle_lib):
    o = oracle_lib
    for x, code in [(1.375, 0x3e), (250.0, 0x5c), (300.0, 0x5d), (-240.0, 0xdc), (1.0, 0x3c)]:
        assert o.encode(x, E5M2) == code, x
    assert o.decode(0x3e, E5M2) == 1.5
    assert o.decode(0x5c, E5M2) == 256.0
    assert o.decode(0x5d, E5M2) == 320.0
    assert o.decode(0xdc, E5M2) == -256.0


def test_format_constants(oracle_lib):
    o = oracle_lib
    assert o.lib().orc_max_finite(E4M3) == 240.0
    assert o.lib().orc_max_finite(E5M2) == 57344.0
    assert math.isinf(o.decode(0x78, E4M3))
    assert math.isnan(o.decode(0x7f, E4M3))


def test_every_code_round_trips_through_the_encoder(oracle_lib):
    o = oracle_lib
    for fmt in (E4M3, E5M2):
        for code in range(256):
            v = o.decode(code, fmt)
            if not math.isfinite(v):
                continue
            assert o.encode(v, fmt) == code, (fmt, hex(code), v)


def test_rounding_is_to_nearest_even(oracle_lib):
    o = oracle_lib
    assert o.encode(1.0625, E4M3) == 0x38
    assert o.encode(1.1875, E4M3) == 0x3a
    assert o.encode(1.0626, E4M3) == 0x39


def test_per_channel_scales_stretch_each_row_to_full_scale(oracle_lib):
    o = oracle_lib
    w = bf(o, [0.5, -1.0, 0.25, 0.0, 100.0, -50.0, 12.5, 0.0])
    codes, scales, bias = o.quantize(w, 2, 4, E4M3, PCS)
    assert scales[0] == np.float32(1.0) / np.float32(240.0)
    assert scales[1] == np.float32(100.0) / np.float32(240.0)
    assert bias == 7
    assert codes[1] & 0x7f == 0x77 and codes[4] & 0x7f == 0x77
    d = o.dequantize(codes, scales, 2, 4, E4M3)
    assert abs(d[0] - 0.5) < 0.5 * 0.07 and abs(d[4] - 100.0) < 100.0 * 0.07


def test_hw_exp_bias_picks_the_finest_range_that_fits(oracle_lib):
    o = oracle_lib
    ch = o.lib().orc_choose_exp_bias
    assert [ch(x, E4M3) for x in (0.5, 0.9375, 1.0, 15.0, 16.0, 1000.0, 1e9)] == \
        [15, 15, 11, 11, 7, 3, 3]
    assert ch(1e9, E5M2) == 15
    w = bf(o, [(i - 32.0) / 64.0 for i in range(64)])
    codes, scales, bias = o.quantize(w, 4, 16, E4M3, HW)
    assert bias == 15 and np.all(scales == np.float32(1.0 / 256.0))


def test_unit_scaling_leaves_the_codes_alone(oracle_lib):
    o = oracle_lib
    w = bf(o, [1.0, 2.0, 0.5, 100.0])
    codes, scales, _ = o.quantize(w, 1, 4, E4M3, UNIT)
    assert list(scales) == [1.0]
    assert codes[0] == o.encode(1.0, E4M3) and codes[3] == o.encode(100.0, E4M3)


def test_dequantize_of_quantize_is_within_the_format_resolution(oracle_lib):
    o = oracle_lib
    rows, cols = 32, 128
    i = np.arange(rows * cols, dtype=np.uint64)
    x = ((i * 2654435761) % 65536).astype(np.float32) / np.float32(65536.0) - np.float32(0.5)
    x = x * (np.float32(1.0) + (i // cols).astype(np.float32))
    w = bf(o, x)
    codes, scales, _ = o.quantize(w, rows, cols, E4M3, PCS)
    mean, mx = o.row_errors(w, codes, scales, rows, cols, E4M3)
    assert np.all(mx <= 0.0626) and np.all(mean < 0.03)


def _ramp(o, rows, cols):
    i = np.arange(rows * cols, dtype=np.int64)
    x = (((i * 7919) % 2003).astype(np.float32) - np.float32(1000.0)) / np.float32(977.0)
    return bf(o, x)


def test_the_parallel_path_agrees_with_the_serial_one(oracle_lib):
    o = oracle_lib
    rows, cols = 512, 4096
    w = _ramp(o, rows, cols)
    assert o.lib().orc_split(rows, cols) > 1
    par = o.quantize(w, rows, cols, E4M3, PCS)
    ser = o.quantize(w, rows, cols, E4M3, PCS, threads=1)
    assert np.array_equal(par[0], ser[0]) and np.array_equal(par[1], ser[1])


def test_the_parallel_path_carries_a_ragged_last_chunk(oracle_lib):
    o = oracle_lib
    rows, cols = 67, 16 * 1024
    w = _ramp(o, rows, cols)
    t = o.lib().orc_split(rows, cols)
    assert t > 1 and rows % t != 0
    for s in (PCS, HW, UNIT):
        par = o.quantize(w, rows, cols, E4M3, s)
        ser = o.quantize(w, rows, cols, E4M3, s, threads=1)
        assert np.array_equal(par[0], ser[0]), s
        assert np.any(par[0][(rows - 1) * cols:] != 0), s


def test_the_hardware_bias_scheme_is_the_identity_for_e5m2(oracle_lib):
    o = oracle_lib
    i = np.arange(4 * 32)
    w = bf(o, (((i * 37) % 101) - 50.0) / 13.0)
    hw = o.quantize(w, 4, 32, E5M2, HW)
    unit = o.quantize(w, 4, 32, E5M2, UNIT)
    assert hw[2] == 15 and np.all(hw[1] == 1.0) and np.array_equal(hw[0], unit[0])


def test_zero_rows_keep_a_unit_scale(oracle_lib):
    o = oracle_lib
    codes, scales, _ = o.quantize(np.zeros(8, np.uint16), 2, 4, E4M3, PCS)
    assert list(scales) == [1.0, 1.0] and not codes.any()
    mean, mx = o.row_errors(np.zeros(8, np.uint16), codes, scales, 2, 4, E4M3)
    assert mean[0] == 0.0 and mx[0] == 0.0


def test_a_backoff_leaves_headroom(oracle_lib):
    o = oracle_lib
    w = bf(o, [1.0, -0.5, 0.25, 0.125])
    codes, scales, _ = o.quantize(w, 1, 4, E4M3, PCS, backoff=0.5)
    assert scales[0] == np.float32(1.0) / np.float32(120.0)
    assert codes[0] == 0x6f and o.decode(codes[0], E4M3) == 120.0


def test_bad_arguments_are_refused(oracle_lib):
    o = oracle_lib
    with pytest.raises(ValueError):
        o.quantize(np.zeros(0, np.uint16), 0, 0, E4M3, PCS)
    with pytest.raises(ValueError):
        o.quantize(np.zeros(4, np.uint16), 1, 4, E4M3, PCS, backoff=0.0)


# ------------------------------------------------------------- golden file --

def test_the_fixture_is_the_one_the_generator_writes():
    doc, cases = load_cases()
    assert doc["generator"] == "tools/fp8_fixtures.py"
    assert len(cases) >= 12
    assert sum(c["name"].startswith("ckpt_") for c in cases) >= 6


def test_scales_and_codes_match_the_golden_file(oracle_lib):
    o = oracle_lib
    _, cases = load_cases()
    for c in cases:
        codes, scales, bias = o.quantize(c["w"], c["rows"], c["cols"], FMT[c["format"]],
                                         SCL[c["scaling"]])
        assert bias == c["exp_bias"], c["name"]
        assert np.array_equal(scales.view(np.uint32), c["scales"]), c["name"]
        assert np.array_equal(codes, c["codes"]), c["name"]


def test_the_only_divergence_from_torch_is_the_saturation(oracle_lib):
    o = oracle_lib
    _, cases = load_cases()
    checked = 0
    for c in cases:
        if "torch_raw" not in c:
            continue
        checked += 1
        fmt = FMT[c["format"]]
        codes, _, _ = o.quantize(c["w"], c["rows"], c["cols"], fmt, SCL[c["scaling"]])
        reserved = 0x78 if fmt == E4M3 else 0x7c
        maxc = 0x77 if fmt == E4M3 else 0x7b
        raw = c["torch_raw"]
        sat = (raw & reserved) == reserved
        assert sat.any(), c["name"]
        assert np.array_equal(codes[sat], (raw[sat] & 0x80) | maxc), c["name"]
        assert np.array_equal(codes[~sat], raw[~sat]), c["name"]
    assert checked >= 2


def test_row_error_statistics_match_numpy(oracle_lib):
    o = oracle_lib
    _, cases = load_cases()
    for c in cases:
        fmt = FMT[c["format"]]
        codes, scales, _ = o.quantize(c["w"], c["rows"], c["cols"], fmt, SCL[c["scaling"]])
        mean, mx = o.row_errors(c["w"], codes, scales, c["rows"], c["cols"], fmt)
        for r in range(c["rows"]):
            wm, wx = c["mean_rel"][r], c["max_rel"][r]
            assert abs(float(mean[r]) - wm) <= 1e-6 + 1e-5 * wm, (c["name"], r)
            assert abs(float(mx[r]) - wx) <= 1e-6 + 1e-5 * wx, (c["name"], r)


def test_checkpoint_rows_quantize_within_the_formats_resolution(oracle_lib):
    o = oracle_lib
    _, cases = load_cases()
    seen = 0
    for c in cases:
        if not c["name"].startswith("ckpt_") or c["scaling"] != "pcs":
            continue
        seen += 1
        rows, cols = c["rows"], c["cols"]
        codes, scales, _ = o.quantize(c["w"], rows, cols, E4M3, PCS)
        mean, mx = o.row_errors(c["w"], codes, scales, rows, cols, E4M3)
        assert np.all(mean < 0.03) and np.all(mx <= 0.25), c["name"]
        back = o.dequantize(codes, scales, rows, cols, E4M3).reshape(rows, cols)
        wf = (c["w"].astype(np.uint32) << 16).view(np.float32).reshape(rows, cols)
        for r in range(rows):
            ai = int(np.argmax(np.abs(wf[r])))
            assert abs(back[r, ai] - wf[r, ai]) <= abs(wf[r, ai]) * 1e-6, (c["name"], r)
    assert seen >= 3


def test_an_infinite_weight_gives_the_x86_default_nan(oracle_lib):
    """An inf in a row makes its scale inf; +-inf / inf is a NaN the division
    generates, which on x86 (where the reference runs) is the negative
    'real indefinite': both infinities encode to 0xff, finite weights to
    signed zero."""
    o = oracle_lib
    w = bf(o, [math.inf, -math.inf, 1.0, -2.0])
    codes, scales, _ = o.quantize(w, 1, 4, E4M3, PCS)
    assert math.isinf(scales[0])
    assert list(codes) == [0xff, 0xff, 0x00, 0x80]

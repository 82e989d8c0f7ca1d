"""GPU parity of the FP8 quantizer (K11): bit-exact codes, scales and exponent
bias against the CPU oracle (itself pinned to the reference's golden file),
through the C ABI, on the golden cases, the config-0 matrix and ragged shapes,
plus the encoder over all 2^32 f32 inputs."""
import numpy as np
import pytest

from test_fp8_oracle import FMT, SCL, load_cases

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fp8(reng_lib):
    from reng import fp8
    return fp8


def test_golden_cases_bit_exact_on_the_gpu(fp8, oracle_lib):
    _, cases = load_cases()
    for c in cases:
        q = fp8.quantize(c["w"], c["rows"], c["cols"], FMT[c["format"]], SCL[c["scaling"]])
        assert q.exp_bias == c["exp_bias"], c["name"]
        assert np.array_equal(q.scales.view(np.uint32), c["scales"]), c["name"]
        assert np.array_equal(q.codes, c["codes"]), c["name"]


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("scaling", [0, 1, 2])
def test_config0_matrix_bit_exact_device_memory(fp8, oracle_lib, fmt, scaling):
    import torch
    from reng.synth import fp8_config0_matrix
    rows = cols = 4096
    w = fp8_config0_matrix(rows, cols, seed=1234)
    codes_o, scales_o, bias_o = oracle_lib.quantize(w, rows, cols, fmt, scaling)
    wd = torch.from_numpy(w.view(np.int16)).cuda()
    codes, scales, bias = fp8.quantize_device(wd, rows, cols, fmt, scaling)
    torch.cuda.synchronize()
    assert bias == bias_o
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), scales_o.view(np.uint32))
    got = codes.cpu().numpy().reshape(-1)
    bad = np.flatnonzero(got != codes_o)
    assert bad.size == 0, (bad[:4], got[bad[:4]], codes_o[bad[:4]])
    # per-channel scaling puts every row's absmax on the largest finite code
    if scaling == 0:
        assert np.count_nonzero((codes_o & 0x7f) == (0x77 if fmt == 0 else 0x7b)) >= rows


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("cols", [4096, 8192])
def test_every_bf16_value_under_many_row_scales(fp8, oracle_lib, fmt, cols):
    """Per-channel scaling of rows [A, every finite bf16 x with |x| < A]
    for 48 absmax values A with awkward mantissas: the device forms most
    codes from x * RN(1/s) and falls back to IEEE division near the
    format's rounding boundaries; every code and scale must equal the
    oracle's x / s (both the warp-per-row and the CTA-per-row kernels)."""
    import torch
    rng = np.random.default_rng(77 + fmt + cols)
    bits = np.arange(1 << 16, dtype=np.uint32)
    finite = bits[((bits >> 7) & 0xff) != 0xff].astype(np.uint16)
    mag = (finite.astype(np.uint32) << 16).view(np.float32)
    rows = []
    for _ in range(48):
        e = int(rng.integers(-20, 21))
        a = np.float32(np.ldexp(1.0 + rng.integers(1, 128) / 128.0, e))
        a_bits = np.uint16(a.view(np.uint32) >> 16)
        a = (np.uint32(a_bits) << 16).view(np.float32)
        body = finite[np.abs(mag) < a]
        chunk = cols - 1
        for i in range(0, body.size, chunk):
            r = np.zeros(cols, np.uint16)
            r[0] = a_bits
            part = body[i:i + chunk]
            r[1:1 + part.size] = part
            rows.append(r)
    w = np.stack(rows)
    n = w.shape[0]
    codes_o, scales_o, _ = oracle_lib.quantize(w.reshape(-1), n, cols, fmt, 0)
    codes, scales, _ = fp8.quantize_device(torch.from_numpy(w.view(np.int16)).cuda(), n, cols, fmt, 0)
    torch.cuda.synchronize()
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), scales_o.view(np.uint32))
    got = codes.cpu().numpy().reshape(-1)
    bad = np.flatnonzero(got != codes_o)
    assert bad.size == 0, (bad.size, bad[:4], got[bad[:4]], codes_o[bad[:4]])


def _special_row(rng, cols):
    x = rng.standard_normal(cols).astype(np.float32)
    sp = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -1e-40, 3e38, 240.0, 248.0,
                   -247.9, 57344.0, 61440.0, 2.0 ** -9, 2.0 ** -10, 1.5 * 2.0 ** -10],
                  np.float32)
    k = min(cols, sp.size)
    x[:k] = sp[:k]
    return x


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 7), (5, 8), (67, 1000), (2, 20000),
                                       (9, 4104), (1, 16384)])
def test_ragged_and_special_values(fp8, oracle_lib, rows, cols):
    from reng.synth import f32_to_bf16_bits
    rng = np.random.default_rng(rows * 1000 + cols)
    x = np.concatenate([_special_row(rng, cols) for _ in range(rows)])
    w = f32_to_bf16_bits(x)
    for fmt in (0, 1):
        for scaling in (0, 1, 2):
            co, so, bo = oracle_lib.quantize(w, rows, cols, fmt, scaling)
            q = fp8.quantize(w, rows, cols, fmt, scaling)
            assert q.exp_bias == bo
            assert np.array_equal(q.scales.view(np.uint32), so.view(np.uint32)), (fmt, scaling)
            assert np.array_equal(q.codes, co), (fmt, scaling)


def test_zero_rows_and_backoff_on_the_gpu(fp8):
    q = fp8.quantize(np.zeros(8, np.uint16), 2, 4, 0, 0)
    assert list(q.scales) == [1.0, 1.0] and not q.codes.any()
    from reng.synth import f32_to_bf16_bits
    w = f32_to_bf16_bits(np.array([1.0, -0.5, 0.25, 0.125], np.float32))
    q = fp8.quantize_with(w, 1, 4, 0, 0, 0.5)
    assert q.scales[0] == np.float32(1.0) / np.float32(120.0) and q.codes[0] == 0x6f


def test_bad_arguments_raise(fp8):
    with pytest.raises(ValueError):
        fp8.quantize(np.zeros(4, np.uint16), 0, 4, 0, 0)
    with pytest.raises(ValueError):
        fp8.quantize_with(np.zeros(4, np.uint16), 1, 4, 0, 0, float("nan"))


@pytest.mark.parametrize("fmt", [0, 1])
def test_encoder_equals_the_oracle_on_every_f32(reng_lib, oracle_lib, fmt):
    """All 2^32 f32 bit patterns, compared by per-chunk checksums."""
    import torch
    chunk = 1 << 28
    w = (torch.arange(1 << 16, device="cuda", dtype=torch.int64) + 1)
    codes = torch.empty(chunk, dtype=torch.uint8, device="cuda")
    for c in range(1 << 32 >> 28):
        lo = c * chunk
        x = torch.arange(lo, lo + chunk, device="cuda", dtype=torch.int64).to(torch.int32)
        reng_lib.call("reng_fp8_encode", x.data_ptr(), chunk, fmt, codes.data_ptr(),
                      torch.cuda.current_stream().cuda_stream)
        got = int((codes.view(-1, 1 << 16).to(torch.int64) * w).sum().item())
        want = oracle_lib.encode_checksum(lo, lo + chunk, fmt)
        assert got == want, "chunk %d (f32 bits 0x%08x..)" % (c, lo)


def test_decode_matches_the_oracle(reng_lib, oracle_lib):
    import torch
    for fmt in (0, 1):
        codes = torch.arange(256, dtype=torch.int32).to(torch.uint8).cuda()
        out = torch.empty(256, dtype=torch.float32, device="cuda")
        reng_lib.call("reng_fp8_decode", codes.data_ptr(), 256, fmt, out.data_ptr(),
                      torch.cuda.current_stream().cuda_stream)
        got = out.cpu().numpy()
        want = np.array([oracle_lib.decode(c, fmt) for c in range(256)], np.float32)
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(got), nan)
        assert np.array_equal(got[~nan], want[~nan])


@pytest.mark.parametrize("product", ["1", "0"])
@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("scaling", [0, 2])
def test_both_quotient_paths_are_bit_exact(fp8, oracle_lib, monkeypatch, fmt, scaling, product):
    """The default division-free quotient (Markstein's correction of
    x * RN(1/s), csrc/fp8_product.h) and the IEEE division it replaces
    (RENG_FP8_PRODUCT=0): the config-0 matrix and the rows of special
    values, bit for bit against the oracle's x / s."""
    import torch
    from reng.synth import f32_to_bf16_bits, fp8_config0_matrix
    monkeypatch.setenv("RENG_FP8_PRODUCT", product)
    rows = cols = 4096
    w = fp8_config0_matrix(rows, cols, seed=99)
    co, so, bo = oracle_lib.quantize(w, rows, cols, fmt, scaling)
    codes, scales, bias = fp8.quantize_device(torch.from_numpy(w.view(np.int16)).cuda(), rows, cols, fmt, scaling)
    torch.cuda.synchronize()
    assert bias == bo
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), so.view(np.uint32))
    got = codes.cpu().numpy().reshape(-1)
    bad = np.flatnonzero(got != co)
    assert bad.size == 0, (bad[:4], got[bad[:4]], co[bad[:4]])
    rng = np.random.default_rng(5)
    x = np.concatenate([_special_row(rng, 4104) for _ in range(9)])
    ws = f32_to_bf16_bits(x)
    co, so, bo = oracle_lib.quantize(ws, 9, 4104, fmt, scaling)
    q = fp8.quantize(ws, 9, 4104, fmt, scaling)
    assert np.array_equal(q.scales.view(np.uint32), so.view(np.uint32))
    assert np.array_equal(q.codes, co)


@pytest.mark.parametrize("product", ["0", "1"])
def test_a_negative_nan_weight_keeps_its_sign(fp8, oracle_lib, monkeypatch, product):
    """The reference's x86 division returns a NaN operand as it is, sign
    included: a negative NaN weight encodes to 0xff, a positive one to 0x7f
    (division and division-free paths)."""
    monkeypatch.setenv("RENG_FP8_PRODUCT", product)
    w = np.array([0x3F80, 0xFFC0, 0x7FC0, 0xBF00, 0x4000, 0x0000, 0x8000, 0x3E00] * 2, np.uint16)
    for fmt in (0, 1):
        co, so, _ = oracle_lib.quantize(w, 2, 8, fmt, 0)
        q = fp8.quantize(w, 2, 8, fmt, 0)
        assert co[1] == 0xFF and co[2] == 0x7F
        assert np.array_equal(q.codes, co), (fmt, q.codes, co)

"""The CPU oracle (and the reference build) against the reference's own pinned
vectors, extracted from its C tests into tests/golden/pins.json."""
import numpy as np
import pytest


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def libs(oracle, request):
    out = [("oracle", oracle)]
    from oracle.oracle import REF_SO, Reference
    if REF_SO.exists():
        out.append(("reference", Reference()))
    return out


def test_gelu_hex_pin(oracle, pins, request):
    p = pins["gelu_hex"]
    for name, lib in libs(oracle, request):
        ok, y = lib.erf_gelu(np.array(p["input"], np.float32))
        assert ok and list(bits(y)) == p["expected_bits"], name


def test_gelu_closed_form(oracle, pins):
    p = pins["gelu_closed_form"]
    ok, y = oracle.erf_gelu(np.array(p["input"], np.float32))
    assert ok and np.allclose(y, p["expected"], atol=p["atol"], rtol=0)


def test_layer_norm_regression_bits(oracle, pins, request):
    p = pins["layer_norm_regression"]
    x = np.array(p["input_bits"], np.uint32).view(np.float32)
    for name, lib in libs(oracle, request):
        ok, y = lib.layer_norm(x, np.ones(512, np.float32), np.zeros(512, np.float32))
        assert ok and bits(y)[0] == p["expected_first_bits"], name


def test_layer_norm_closed_form(oracle):
    # tests/test_phonon_transformer.c:547-551
    x = np.array([1.0, -2.0, 3.0], np.float32)
    ok, y = oracle.layer_norm(x, np.array([1.0, 2.0, 0.5], np.float32),
                              np.array([0.0, 0.1, -0.1], np.float32))
    d = np.sqrt(np.float32(38.0 / 9.0) + np.float32(1e-5))
    assert ok
    assert abs(y[0] - (1 / 3) / d) < 1e-5
    assert abs(y[1] - ((-8 / 3) / d * 2 + 0.1)) < 1e-5
    assert abs(y[2] - ((7 / 3) / d * 0.5 - 0.1)) < 1e-5


def test_rms_norm_closed_form(oracle):
    x = np.array([1.0, -2.0, 3.0], np.float32)
    ok, y = oracle.rms_norm(x, np.array([2.0, 0.5, -1.0], np.float32))
    inv = 1.0 / np.sqrt(14.0 / 3.0 + 1e-5)
    assert ok and np.allclose(y, [2 * inv, -inv, -3 * inv], atol=1e-6, rtol=0)


@pytest.mark.parametrize("case", range(5))
def test_attention_regression_bits(oracle, pins, request, case):
    c = pins["attention_regression"]["cases"][case]
    n = c["count"]
    q = np.zeros(64, np.float32)
    q[0] = 8
    k = np.zeros(n * 64, np.float32)
    v = np.zeros(n * 64, np.float32)
    k[0] = 2
    k[(n - 1) * 64] = c["tail"]
    v[0] = v[(n - 1) * 64] = 0.01
    if c["middle"]:
        k[512 * 64] = c["middle"]
    for name, lib in libs(oracle, request):
        ok, out = lib.attention(q, k, v, n, 64)
        assert ok and bits(out)[0] == c["expected_bits"], name
        assert np.all(out[1:] == 0)


def test_rope_hf_pins(oracle, pins, request):
    p = pins["rope_hf"]
    for pos, exp in zip(p["positions"], p["expected"]):
        row = np.zeros(64, np.float32)
        row[2], row[3] = 1.0, -0.5
        for name, lib in libs(oracle, request):
            ok, y = lib.rope(row, 1, pos, p["theta"])
            assert ok and abs(y[2] - exp[0]) < p["atol"] and abs(y[3] - exp[1]) < p["atol"], name


def test_rope_small_head(oracle):
    # tests/test_phonon_transformer.c:564-569, scalar libm tail (2 frequencies)
    ok, y = oracle.rope(np.array([1, 0, 0, 1], np.float32), 1, 1)
    assert ok
    assert abs(y[0] - np.cos(1.0)) < 1e-6 and abs(y[1] - np.sin(1.0)) < 1e-6
    assert abs(y[2] + np.sin(0.01)) < 1e-6 and abs(y[3] - np.cos(0.01)) < 1e-6
    ok, _ = oracle.rope(np.zeros(4, np.float32), 3, 0)
    assert not ok


def test_sleef_sincos_pins(pins, request):
    from oracle.oracle import REF_SO, Reference
    if not REF_SO.exists():
        pytest.skip("reference build absent")
    p = pins["sleef_math"]
    c, s = Reference().sincos(np.array(p["phases"], np.float32))
    assert list(bits(c)) == p["cos_expected_bits"]
    assert list(bits(s)) == p["sin_expected_bits"]


def _block(scale, values):
    b = np.zeros(34, np.uint8)
    b[0], b[1] = scale & 0xFF, scale >> 8
    b[2:] = np.asarray(values, np.int8).view(np.uint8)
    return b


def test_q8_known_answers(oracle, request):
    # tests/test_phonon_q8.c:9-55
    b0 = _block(0x3800, np.arange(32) - 16)
    b1 = _block(0x4000, np.ones(32))
    ones = np.ones(64, np.float32)
    for name, lib in libs(oracle, request):
        ok, v = lib.q8_dot(np.concatenate([b0, b1]), ones)
        assert ok and v == 56.0, name
        ok, out = lib.q8_matvec(np.concatenate([b0, b1, b1, b0]), ones, 2, 64)
        assert ok and list(out) == [56.0, 56.0], name
        rows = np.concatenate([_block(0x3800, np.ones(32)), _block(0x4000, 2 * np.ones(32)),
                               _block(0x3800, -np.ones(32)), _block(0x4000, 3 * np.ones(32))])
        x = np.concatenate([np.ones(32), 2 * np.ones(32)]).astype(np.float32)
        ok, out = lib.q8_matvec(rows, x, 2, 64)
        assert ok and list(out) == [272.0, 368.0], name
        ok, v = lib.q8_dot(_block(0x0001, np.ones(32)), np.ones(32, np.float32))
        assert ok and v == 2.0 ** -19, name
        ok, _ = lib.q8_dot(_block(0x7C00, np.ones(32)), np.ones(32, np.float32))
        assert not ok, name
        x = np.ones(32, np.float32)
        x[0] = np.inf
        ok, _ = lib.q8_dot(_block(0x0001, np.ones(32)), x)
        assert not ok, name


def test_linear_edges(oracle, pins, request):
    p = pins["linear_edges"]
    for name, lib in libs(oracle, request):
        ok, y = lib.linear(2, np.array(p["bf16_2x2"]["weights"], np.uint16), 2, 2,
                           np.array(p["bf16_2x2"]["input"], np.float32))
        assert ok and list(y) == p["bf16_2x2"]["expected"], name
        q8 = np.concatenate([_block(0x0001, np.ones(32)), _block(0x8000, np.ones(32))])
        ok, y = lib.linear(1, q8, 2, 32, np.ones(32, np.float32))
        assert ok and list(y) == p["q8_scale_edges"]["expected"], name
        for bad in p["q8_scale_edges"]["rejected_scales"]:
            q8 = np.concatenate([_block(bad, np.ones(32)), _block(0x3C00, np.ones(32))])
            ok, _ = lib.linear(1, q8, 2, 32, np.ones(32, np.float32))
            assert not ok, name


def test_linear_cancellation_pin_reference_only(reference, pins):
    """[1e8,1,-1e8,1] x ones: Accelerate's SGEMM order gives [0, 0.25]. The
    value depends on the BLAS reduction order; it is recorded here for the
    OpenBLAS build rather than asserted for every implementation."""
    x = np.array([1e8 if i % 4 == 0 else (-1e8 if i % 4 == 2 else 1.0) for i in range(32)],
                 np.float32)
    ok, y = reference.linear(2, np.full(64, 0x3F80, np.uint16), 2, 32, x,
                             bias=np.array([0.0, 0.25], np.float32))
    assert ok
    assert np.all(np.isfinite(y))


def test_sleef_table_row_sums_to_inv_2pi():
    """The rempif row restated in oracle/sleef_u10.c splits 1/(2 pi)."""
    from decimal import Decimal, getcontext
    getcontext().prec = 60
    pi = Decimal("3.14159265358979323846264338327950288419716939937510582097494")
    pieces = [0.159154892, 5.112411827e-08, 3.626141271e-15, -2.036222915e-22]
    total = sum(Decimal(float(np.float32(p))) for p in pieces)
    assert abs(total - 1 / (2 * pi)) < Decimal("1e-28")

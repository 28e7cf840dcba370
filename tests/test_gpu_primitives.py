"""GPU primitives and linears against the CPU oracle and the reference pins."""
import numpy as np
import pytest

from phonon_b200 import runtime as rt
from phonon_b200 import synth

pytestmark = pytest.mark.gpu


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_layer_norm_bit_exact(cuda_ok, oracle, pins):
    p = pins["layer_norm_regression"]
    x = np.array(p["input_bits"], np.uint32).view(np.float32)
    one, zero = np.ones(512, np.float32), np.zeros(512, np.float32)
    rc, y = rt.layer_norm(x, one, zero)
    assert rc == rt.OK and bits(y)[0] == p["expected_first_bits"]
    g = synth.Generator(21)
    for scale in (1e-3, 1.0, 37.0):
        x = g.normal(512) * scale
        w, b = g.normal(512) * 0.1 + 1, g.normal(512) * 0.1
        rc, y = rt.layer_norm(x, w, b)
        ok, yo = oracle.layer_norm(x, w, b)
        assert rc == rt.OK and ok and np.array_equal(bits(y), bits(yo))


def test_layer_norm_other_widths_and_failures(cuda_ok, oracle):
    x = np.array([1.0, -2.0, 3.0], np.float32)
    w, b = np.array([1.0, 2.0, 0.5], np.float32), np.array([0.0, 0.1, -0.1], np.float32)
    rc, y = rt.layer_norm(x, w, b)
    ok, yo = oracle.layer_norm(x, w, b)
    assert rc == rt.OK and np.array_equal(bits(y), bits(yo))
    x512 = np.ones(512, np.float32)
    x512[7] = np.nan
    rc, _ = rt.layer_norm(x512, np.ones(512, np.float32), np.zeros(512, np.float32))
    assert rc == rt.NON_FINITE


def test_gelu_bit_exact(cuda_ok, oracle, pins):
    p = pins["gelu_hex"]
    rc, y = rt.erf_gelu(np.array(p["input"], np.float32))
    assert rc == rt.OK and list(bits(y)) == p["expected_bits"]
    x = synth.Generator(3).normal(4096) * 4
    rc, y = rt.erf_gelu(x)
    ok, yo = oracle.erf_gelu(x)
    assert rc == rt.OK and np.array_equal(bits(y), bits(yo))
    rc, y = rt.erf_gelu(x[:7])  # scalar tail (erf in double vs libm erff)
    ok, yo = oracle.erf_gelu(x[:7])
    assert rc == rt.OK and rt.rel_err(y, yo) < 1e-6


def test_rope_pins_and_oracle(cuda_ok, oracle, pins):
    p = pins["rope_hf"]
    for pos, exp in zip(p["positions"], p["expected"]):
        row = np.zeros(64, np.float32)
        row[2], row[3] = 1.0, -0.5
        rc, y = rt.rope(row, 1, pos)
        assert rc == rt.OK and abs(y[2] - exp[0]) < p["atol"] and abs(y[3] - exp[1]) < p["atol"]
    x = synth.Generator(8).normal(512)
    for pos in (0, 5, 139, 4095, 8191):
        rc, y = rt.rope(x, 8, pos)
        ok, yo = oracle.rope(x, 8, pos)
        assert rc == rt.OK and rt.rel_err(y, yo) < 1e-5  # cos/sin rounded from double vs SLEEF u10


def _block(scale, values):
    b = np.zeros(34, np.uint8)
    b[0], b[1] = scale & 0xFF, scale >> 8
    b[2:] = np.asarray(values, np.int8).view(np.uint8)
    return b


def test_q8_known_answers(cuda_ok):
    b0 = _block(0x3800, np.arange(32) - 16)
    b1 = _block(0x4000, np.ones(32))
    assert rt.Linear(np.concatenate([b0, b1]), 1, 64)(np.ones(64))[0, 0] == 56.0
    y = rt.Linear(np.concatenate([b0, b1, b1, b0]), 2, 64)(np.ones(64))
    assert list(y[0]) == [56.0, 56.0]
    rows = np.concatenate([_block(0x3800, np.ones(32)), _block(0x4000, 2 * np.ones(32)),
                           _block(0x3800, -np.ones(32)), _block(0x4000, 3 * np.ones(32))])
    x = np.concatenate([np.ones(32), 2 * np.ones(32)])
    assert list(rt.Linear(rows, 2, 64)(x)[0]) == [272.0, 368.0]
    q8 = np.concatenate([_block(0x0001, np.ones(32)), _block(0x8000, np.ones(32))])
    assert list(rt.Linear(q8, 2, 32)(np.ones(32))[0]) == [2.0 ** -19, 0.0]
    for bad in (0x7C00, 0x7E00):
        with pytest.raises(rt.CudaError) as e:
            rt.Linear(np.concatenate([_block(bad, np.ones(32)), b1[:34]]), 2, 32)
        assert e.value.status == rt.NON_FINITE
    x = np.ones(32)
    x[3] = np.inf
    with pytest.raises(rt.CudaError):
        rt.Linear(_block(0x3C00, np.ones(32)), 1, 32)(x)


def test_bf16_linear_pin(cuda_ok):
    lin = rt.Linear(np.array([0x3F80, 0xC000, 0x4000, 0x3F00], np.uint16), 2, 2, kind=rt.BF16)
    assert list(lin(np.array([3.0, 2.0]))[0]) == [-1.0, 7.0]


@pytest.mark.parametrize("scale_mode", [synth.SCALE_PER_LINEAR, synth.SCALE_PER_ROW])
def test_flow_linears_vs_oracle(cuda_ok, oracle, scale_mode):
    g = synth.Generator(31 + scale_mode)
    for rows, cols in ((1536, 512), (512, 512), (2048, 512), (512, 2048)):
        w = g.q8_linear(rows, cols, scale_mode)
        lin = rt.Linear(w, rows, cols)
        assert lin.bytes() == rows * cols // 32 * 34
        for batch in (1, 8, 64):
            x = g.normal(batch * cols)
            y = lin(x).ravel()
            ok, yo = oracle.linear(1, w, rows, cols, x, batch)
            assert ok and rt.rel_err(y, yo) < 1e-4
            assert np.abs(y - yo).max() / np.abs(yo).max() < 1e-5

"""The C restatement against the unmodified reference (oracle/_ref) on the
seeded 12-layer model: bit-exact primitives, teacher-forced per-layer error
<= 1e-4 and chained final-layer error <= 1e-3.

Error metric (all parity tests): max_i |a_i - r_i| / max(|r_i|, 1e-2 * max|r|).
A per-element floor at 1e-2 of the vector's largest magnitude is the weakest
floor at which two correct fp32 implementations that only reorder sums (this
restatement vs OpenBLAS SGEMM) meet the 1e-4 per-layer bound; with a 1e-6
floor they differ by ~7e-3 on near-zero elements."""
import numpy as np
import pytest

from phonon_b200 import synth
from phonon_b200.runtime import rel_err

PER_LAYER_TOL = 1e-4
FINAL_TOL = 1e-3


def test_primitives_bit_exact_vs_reference(oracle, reference):
    g = synth.Generator(11)
    for trial in range(20):
        x = (g.normal(512) * (1 + trial)).astype(np.float32)
        w = g.normal(512) * 0.1 + 1
        b = g.normal(512) * 0.1
        assert np.array_equal(oracle.layer_norm(x, w, b)[1], reference.layer_norm(x, w, b)[1])
        assert np.array_equal(oracle.erf_gelu(x * 3)[1], reference.erf_gelu(x * 3)[1])
        for pos in (0, 1, 17, 139, 1000, 8191):
            assert np.array_equal(oracle.rope(x, 8, pos)[1], reference.rope(x, 8, pos)[1])


def test_q8_dot_matvec_bit_exact_vs_reference(oracle, reference):
    g = synth.Generator(5)
    blocks = g.q8_linear(64, 512, synth.SCALE_PER_ROW)
    x = g.normal(512)
    ok1, y1 = oracle.q8_matvec(blocks, x, 64, 512)
    ok2, y2 = reference.q8_matvec(blocks, x, 64, 512)
    assert ok1 and ok2 and np.array_equal(y1, y2)


def test_attention_close_to_reference(oracle, reference):
    g = synth.Generator(9)
    for count in (1, 15, 16, 17, 511, 512, 513, 1300):
        q = g.normal(64)
        k = g.normal(count * 512)
        v = g.normal(count * 512)
        ok1, a = oracle.attention(q, k, v, count, 512)
        ok2, b = reference.attention(q, k, v, count, 512)
        assert ok1 and ok2 and rel_err(a, b) < PER_LAYER_TOL, count


def test_linear_close_to_reference(oracle, reference):
    g = synth.Generator(2)
    for rows, cols in ((1536, 512), (512, 2048)):
        w = g.q8_linear(rows, cols)
        for batch in (1, 8):
            x = g.normal(batch * cols)
            ok1, a = oracle.linear(1, w, rows, cols, x, batch)
            ok2, b = reference.linear(1, w, rows, cols, x, batch)
            assert ok1 and ok2 and rel_err(a, b) < PER_LAYER_TOL


@pytest.fixture(scope="module")
def models(oracle, reference, weights12):
    return oracle.model(weights12), reference.model(weights12)


def test_teacher_forced_layers(models):
    """Each oracle layer gets the reference's layer input and the reference's
    cached K/V for earlier positions."""
    om, rm = models
    cap = 48
    oc, rs = om.new_stream(cap), rm.new_stream(cap)
    n = cap * 512
    okeys = np.ctypeslib.as_array(oc.keys, shape=(12 * n,))
    ovals = np.ctypeslib.as_array(oc.values, shape=(12 * n,))
    g = synth.stream_generator(0, 0)
    worst = 0.0
    for pos in range(40):
        x = g.normal(512)
        ok, _, lo = rm.step(rs, pos, x, layer_outputs=True)
        assert ok
        inp = x
        for layer in range(12):
            ok, yo = om.layer_step(oc, layer, pos, inp)
            assert ok
            worst = max(worst, rel_err(yo, lo[layer]))
            inp = lo[layer]
        for layer in range(12):
            k, v = rm.kv(rs, layer, pos)
            okeys[layer * n + pos * 512: layer * n + pos * 512 + 512] = k
            ovals[layer * n + pos * 512: layer * n + pos * 512 + 512] = v
        oc.length = pos + 1
    om.free_stream(oc)
    rm.free_stream(rs)
    assert worst < PER_LAYER_TOL, worst


def test_chained_final_output(models):
    om, rm = models
    oc, rs = om.new_stream(64), rm.new_stream(64)
    g = synth.stream_generator(0, 1)
    worst = 0.0
    for pos in range(48):
        x = g.normal(512)
        ok1, a, _ = om.step(oc, pos, x)
        ok2, b, _ = rm.step(rs, pos, x)
        assert ok1 and ok2
        worst = max(worst, rel_err(a, b))
    om.free_stream(oc)
    rm.free_stream(rs)
    assert worst < FINAL_TOL, worst


def test_reference_prefill_matches_sequential_steps(oracle, reference, weights12):
    """9-layer model: the reference's batched prefill equals its sequential
    steps within tolerance, which licenses prefilling by steps."""
    w9 = weights12[:9]
    rm = reference.model(w9)
    a, b = rm.new_stream(64), rm.new_stream(64)
    g = synth.stream_generator(3, 0)
    rows = np.stack([g.normal(512) for _ in range(40)])
    out = np.zeros(512, np.float32)
    assert reference.lib.ref_stream_prefill(rm.handle, a, rows.ctypes.data, 40, 10000.0,
                                            out.ctypes.data)
    for pos in range(40):
        ok, y, _ = rm.step(b, pos, rows[pos])
        assert ok
    assert rel_err(y, out) < FINAL_TOL
    for layer in (0, 8):
        ka, va = rm.kv(a, layer, 39)
        kb, vb = rm.kv(b, layer, 39)
        assert rel_err(ka, kb) < FINAL_TOL and rel_err(va, vb) < FINAL_TOL

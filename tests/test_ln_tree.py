"""The device LayerNorm's moment tree equals the reference's cascade, bit for bit.

The kernels (ln_moments512 in speech-mac_b200/csrc/phonon_kernels.cuh) fold
the eight 64-wide chunk results of a warp's row as a balanced tree across
lanes, three shuffle levels, instead of replaying the reference's
binary-counter cascade (src/phonon_transformer.c:90-151) chunk by chunk. The
two orders are the same merges on the same operands: this test restates the
lanes' float32 arithmetic in numpy and compares the mean and 1/sqrt(var+eps)
with the oracle's LayerNorm output bit for bit on random and adversarial rows
(no GPU)."""
import numpy as np
import pytest

F = np.float32


def merge(a_mean, a_m2, mean, m2, c, n):
    delta = F(a_mean - mean)
    mean = F(mean + F(c * delta))
    m2 = F(m2 + F(a_m2 + F(F(F(delta * delta) * c) * n)))
    return mean, m2


def device_moments(x):
    x = np.asarray(x, F)
    lanes = []
    for lane in range(32):
        base = (lane >> 2) * 64 + (lane & 3)
        mean, m2 = F(0), F(0)
        for j in range(16):
            v = x[base + 4 * j]
            delta = F(v - mean)
            mean = F(mean + F(delta * F(F(1) / F(j + 1))))
            m2 = F(m2 + F(delta * F(v - mean)))
        lanes.append([mean, m2])
    for mask, n in ((4, F(16)), (8, F(32)), (16, F(64))):
        nxt = []
        for lane in range(32):
            low = (lane & mask) == 0
            me, ot = lanes[lane], lanes[lane ^ mask]
            acc, add = (me, ot) if low else (ot, me)
            nxt.append(list(merge(add[0], add[1], acc[0], acc[1], F(0.5), n)))
        lanes = nxt
    mu, q = F(0), F(0)
    for k in range(4):  # lanes l = 0..3, 128 samples each: c = 128 / (128 (k + 1)), n = 128 k
        c, n = F(128.0) / F(128.0 * (k + 1)), F(128.0 * k)
        lm, lq = lanes[k]
        delta = F(lm - mu)
        mu = fma32(c, delta, mu)
        prod = F(F(delta * delta) * c)
        q = F(q + fma32(prod, n, lq))
    return mu, q


def fma32(a, b, c):
    """fmaf: the exact a*b + c rounded once to float32 (float64 holds a*b of
    two float32 exactly; the sum is rounded twice only in rare ties, checked
    against the oracle below)."""
    return F(np.float64(a) * np.float64(b) + np.float64(c))


@pytest.mark.parametrize("kind", ["normal", "offset", "spiky", "tiny"])
def test_device_tree_equals_reference_cascade(oracle, kind):
    rng = np.random.default_rng({"normal": 1, "offset": 2, "spiky": 3, "tiny": 4}[kind])
    w = np.ones(512, F)
    b = np.zeros(512, F)
    for _ in range(40):
        x = rng.standard_normal(512).astype(F)
        if kind == "offset":
            x = (x * F(0.01) + F(1000.0)).astype(F)
        elif kind == "spiky":
            x[rng.integers(0, 512, 5)] *= F(1e4)
        elif kind == "tiny":
            x = (x * F(1e-20)).astype(F)
        ok, ref = oracle.layer_norm(x, w, b)
        assert ok
        mu, q = device_moments(x)
        var = F(q * F(1.0 / 512.0))
        scale = F(F(1.0) / F(np.sqrt(np.float64(F(var + F(1e-5))))))
        y = F(F(F(x - mu) * scale) * w) + b
        assert np.array_equal(y.view(np.uint32), ref.view(np.uint32)), kind

"""The seeded generator: algorithm pins against a Python restatement of
splitmix64 / xoshiro256** and exact binary16 / bf16 rounding."""
import numpy as np

from phonon_b200 import synth

M64 = (1 << 64) - 1


def _splitmix(state):
    state = (state + 0x9E3779B97F4A7C15) & M64
    z = state
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return state, z ^ (z >> 31)


def _rotl(v, k):
    return ((v << k) | (v >> (64 - k))) & M64


def _xoshiro(seed, n):
    st, s = seed, []
    for _ in range(4):
        st, z = _splitmix(st)
        s.append(z)
    out = []
    for _ in range(n):
        out.append((_rotl((s[1] * 5) & M64, 7) * 9) & M64)
        t = (s[1] << 17) & M64
        s[2] ^= s[0]
        s[3] ^= s[1]
        s[1] ^= s[2]
        s[0] ^= s[3]
        s[2] ^= t
        s[3] = _rotl(s[3], 45)
    return out


def test_xoshiro_matches_python_restatement():
    for seed in (0, 1, 2, 12345):
        g = synth.Generator(seed)
        assert [g.next_u64() for _ in range(16)] == _xoshiro(seed, 16)


def test_normals_are_standard():
    z = synth.Generator(0).normal(200000)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1) < 0.01


def test_float_to_half_matches_numpy_rne():
    g = np.random.default_rng(0)
    xs = np.concatenate([g.normal(size=2000).astype(np.float32) * 1e-3,
                         np.float32([0.0, -0.0, 6.1e-5, 5.96e-8, 2.98e-8, 65504, 65519, 65520,
                                     1e-9, 3e-5, -3e-5]),
                         g.uniform(0.5, 1.5, 500).astype(np.float32) / 127])
    for x in xs:
        assert synth.float_to_half(float(x)) == int(np.float16(x).view(np.uint16)), x


def test_float_to_bf16_rne():
    g = np.random.default_rng(1)
    xs = g.normal(size=5000).astype(np.float32)
    u = xs.view(np.uint32).astype(np.uint64)
    expect = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    got = np.array([synth.float_to_bf16(float(x)) for x in xs], np.uint16)
    assert np.array_equal(got, expect)


def test_weights_deterministic_and_shaped():
    a = synth.flow_weights(2, seed=0)
    b = synth.flow_weights(2, seed=0)
    c = synth.flow_weights(2, seed=1)
    for k in a[0]:
        assert np.array_equal(a[1][k], b[1][k])
    assert not np.array_equal(a[0]["qkv"], c[0]["qkv"])
    q = a[0]["qkv"].reshape(-1, 34)
    vals = q[:, 2:].view(np.int8)
    assert vals.min() >= -127 and vals.max() <= 127
    scales = q[:, :2].copy().view(np.uint16).ravel()
    assert len(set(scales.tolist())) == 1  # one scale per linear
    s = float(np.uint16(scales[0]).view(np.float16))
    assert 0.5 / (127 * np.sqrt(512)) * 0.99 < s < 1.5 / (127 * np.sqrt(512)) * 1.01
    gamma = synth.bf16_to_float(a[0]["norm1_w"])
    assert abs(gamma.mean() - 1) < 0.01 and 0.01 < gamma.std() < 0.03


def test_per_row_scales():
    blocks = synth.Generator(4).q8_linear(64, 512, synth.SCALE_PER_ROW).reshape(64, 16, 34)
    scales = blocks[:, :, :2].copy().view(np.uint16)[..., 0]
    assert np.all(scales == scales[:, :1])
    assert len(set(scales[:, 0].tolist())) > 32

"""The flow head's CPU oracle, pinned before any GPU kernel is built for it.

The flow head (speech-mac src/phonon_sampler.c:307-393) follows the decode
step in every frame: it turns a transformer output row into the next 32-wide
latent. Its restatement (oracle/flow_head_oracle.c) is pinned here three ways:

- against the golden velocity the reference's own test quotes from an
  independent PyTorch evaluation of a nonzero synthetic head
  (tests/test_phonon_sampler.c:148-197; input formulas restated below, the
  expected vector extracted to tests/golden/pins.json), with the test's own
  2e-4 absolute bound;
- the unmodified reference (oracle/_ref) against the same pin, which checks
  the driver that wraps the arrays in the reference's tensor views;
- restatement against reference on seeded random heads, for forward and for
  the one-step sampler, and in their failure contracts.

The restatement sums its linears sequentially where the reference calls
SGEMM, so the two agree within rounding, not bit for bit."""
import numpy as np
import pytest

from oracle.oracle import HEAD_BLOCKS

# Chained-output bound, as for the transformer stack: two correct fp32
# evaluations that only order their sums differently (sequential vs SGEMM)
# differ by up to ~1.2e-4 after the six residual blocks on these heads.
REL_TOL = 1e-3


def rel_err(a, r):
    a, r = np.asarray(a, np.float64), np.asarray(r, np.float64)
    floor = 1e-2 * np.abs(r).max()
    return float(np.max(np.abs(a - r) / np.maximum(np.abs(r), floor)))


def bf16_trunc(x):
    """float32 -> bf16 bits by dropping the low half (exact for k / 128)."""
    return (np.asarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_round(x):
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def pinned_head():
    """The synthetic head of tests/test_phonon_sampler.c:148-187: every matrix
    is a window into one bf16 array m[i] = ((5i mod 7) - 3) / 128 starting at a
    small offset; biases, gains, norms and time frequencies follow per-slot
    integer patterns."""
    n = 1536 * 512 + 32
    i = np.arange(n)
    m = bf16_trunc(((i * 5) % 7 - 3) / 128.0)

    def mat(rows, cols, offset):
        return np.ascontiguousarray(m[offset:offset + rows * cols].reshape(rows, cols))

    def vec(count, pattern, kind):
        k = np.arange(count)
        if kind in (1, 2):
            v = 1.0 + (((k * 3 + pattern * 5) % 7) - 3) / 128.0
        elif kind == 3:
            v = (k % 8 + 1) / 128.0
        else:
            v = (((k * 3 + pattern * 5) % 11) - 5) / 128.0
        return bf16_trunc(v)

    def lin(rows, cols, offset, pattern):
        return mat(rows, cols, offset), vec(rows, pattern, 0)

    return {
        "input": lin(512, 32, 1, 1), "cond": lin(512, 512, 2, 2),
        "time": [[lin(512, 256, t + 1, t + 3), lin(512, 512, t + 4, t + 5)] for t in range(2)],
        "time_freqs": [vec(128, 30 + t, 3) for t in range(2)],
        "time_alpha": [vec(512, 32 + t, 2) for t in range(2)],
        "block_ada": [lin(1536, 512, b + 3, b + 4) for b in range(HEAD_BLOCKS)],
        "block_norm_w": [vec(512, 10 + b, 1) for b in range(HEAD_BLOCKS)],
        "block_norm_b": [vec(512, 16 + b, 0) for b in range(HEAD_BLOCKS)],
        "block_mlp": [[lin(512, 512, b + 9, b + 10), lin(512, 512, b + 11, b + 12)]
                      for b in range(HEAD_BLOCKS)],
        "final_ada": lin(1024, 512, 22, 23), "final_out": lin(32, 512, 24, 25),
    }


def pinned_inputs():
    i = np.arange(512)
    condition = (((i * 7) % 13) - 6) / 8.0
    j = np.arange(32)
    state = (((j * 11 + 3) % 17) - 8) / 16.0
    return condition.astype(np.float32), state.astype(np.float32)


def random_head(seed):
    rng = np.random.default_rng(seed)

    def lin(rows, cols):
        w = rng.standard_normal((rows, cols)) / np.sqrt(cols)
        return np.ascontiguousarray(bf16_round(w)), bf16_round(0.05 * rng.standard_normal(rows))

    return {
        "input": lin(512, 32), "cond": lin(512, 512),
        "time": [[lin(512, 256), lin(512, 512)] for _ in range(2)],
        "time_freqs": [bf16_round(np.exp(-np.linspace(0, 9, 128))) for _ in range(2)],
        "time_alpha": [bf16_round(1 + 0.1 * rng.standard_normal(512)) for _ in range(2)],
        "block_ada": [lin(1536, 512) for _ in range(HEAD_BLOCKS)],
        "block_norm_w": [bf16_round(1 + 0.1 * rng.standard_normal(512)) for _ in range(HEAD_BLOCKS)],
        "block_norm_b": [bf16_round(0.1 * rng.standard_normal(512)) for _ in range(HEAD_BLOCKS)],
        "block_mlp": [[lin(512, 512), lin(512, 512)] for _ in range(HEAD_BLOCKS)],
        "final_ada": lin(1024, 512), "final_out": lin(32, 512),
    }


def test_oracle_matches_reference_pin(oracle, pins):
    p = pins["flow_head_synthetic"]
    head = pinned_head()
    condition, state = pinned_inputs()
    ok, v = oracle.flow_head_forward(head, condition, state, p["s"], p["t"])
    assert ok
    assert np.max(np.abs(v - np.array(p["expected"], np.float32))) < p["atol"]


def test_reference_build_matches_pin(reference, pins):
    p = pins["flow_head_synthetic"]
    head = pinned_head()
    condition, state = pinned_inputs()
    ok, v = reference.flow_head_forward(head, condition, state, p["s"], p["t"])
    assert ok
    assert np.max(np.abs(v - np.array(p["expected"], np.float32))) < p["atol"]


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_oracle_vs_reference_random_heads(oracle, reference, seed):
    head = random_head(seed)
    rng = np.random.default_rng(100 + seed)
    condition = rng.standard_normal(512).astype(np.float32)
    state = rng.standard_normal(32).astype(np.float32)
    s, t = float(rng.uniform(0, 1)), float(rng.uniform(0, 1))
    ok_o, vo = oracle.flow_head_forward(head, condition, state, s, t)
    ok_r, vr = reference.flow_head_forward(head, condition, state, s, t)
    assert ok_o and ok_r
    assert rel_err(vo, vr) < REL_TOL, rel_err(vo, vr)
    noise = rng.standard_normal(32).astype(np.float32)
    ok_o, yo = oracle.flow_lsd_one_step(head, condition, noise, 0.7)
    ok_r, yr = reference.flow_lsd_one_step(head, condition, noise, 0.7)
    assert ok_o and ok_r
    assert rel_err(yo, yr) < REL_TOL, rel_err(yo, yr)


def test_failure_contracts_agree(oracle, reference):
    head = random_head(5)
    condition = np.ones(512, np.float32)
    state = np.zeros(32, np.float32)
    bad = state.copy()
    bad[3] = np.nan
    for impl in (oracle, reference):
        assert not impl.flow_head_forward(head, condition, bad, 0.0, 1.0)[0]
        assert not impl.flow_head_forward(head, condition, state, float("inf"), 1.0)[0]
        assert not impl.flow_lsd_one_step(head, condition, state, 0.0)[0]  # temperature must be > 0
        assert not impl.flow_lsd_one_step(head, condition, bad, 1.0)[0]
    broken = random_head(5)
    broken["block_norm_w"][2] = broken["block_norm_w"][2].copy()
    broken["block_norm_w"][2][9] = 0x7FC0  # a NaN gain
    for impl in (oracle, reference):
        assert not impl.flow_head_forward(broken, condition, state, 0.0, 1.0)[0]

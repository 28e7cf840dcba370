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

from heads import REL_TOL, pinned_head, pinned_inputs, random_head, rel_err


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

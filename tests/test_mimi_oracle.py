"""The Mimi latent transformer's CPU oracle, pinned before its GPU kernels.

speech-mac's Mimi decoder transformer (src/phonon_mimi.c:108-283) turns each
32-wide latent frame into 16 feature rows: a linear projection, a depthwise
transposed-convolution upsample, and two pre-LayerNorm transformer layers
whose 16 queries per frame attend over a 250-slot ring of keys. Its
restatement (oracle/mimi_oracle.c) is pinned here:

- against the reference test's upsample vectors and its synthetic model,
  whose features the test computes by an independent closed form
  (tests/test_phonon_mimi.c:45-123; restated in tests/mimi_models.py) with
  the test's 4e-6 absolute bound, across the ring's wrap (19 frames = 304
  positions > 250);
- the unmodified reference (oracle/_ref, src/phonon_mimi.c compiled where it
  lies) against the same pins;
- restatement against reference on seeded random models, whole requests and
  frame partitions, within the chained bound 1e-3 (the restatement sums its
  linears sequentially where the reference calls SGEMM);
- their failure contracts."""
import numpy as np
import pytest

import mimi_models
from heads import rel_err

CHAIN_TOL = 1e-3


def _upsample_weight():
    from heads import bf16_trunc
    return np.ascontiguousarray(bf16_trunc(np.arange(1, 9, dtype=np.float32)))  # [2][1][4], k = i + 1


@pytest.mark.parametrize("impl_name", ["oracle", "reference"])
def test_upsample_pins(request, impl_name):
    """tests/test_phonon_mimi.c:45-60: overlap with the previous frame, start-up
    with zeros and the right trim, a non-finite input rejected."""
    impl = request.getfixturevalue(impl_name)
    w = _upsample_weight()
    ok, out = impl.mimi_upsample(w, [2, 3], [5, 7], 2, 2)
    assert ok and out.tolist() == [17, 64, 24, 74]
    ok, out = impl.mimi_upsample(w, [2, 3], [0, 0], 2, 2)
    assert ok and out.tolist() == [2, 15, 4, 18]
    assert not impl.mimi_upsample(w, [np.nan, 3], [0, 0], 2, 2)[0]


@pytest.mark.parametrize("impl_name", ["oracle", "reference"])
def test_synthetic_model_closed_form(request, impl_name):
    impl = request.getfixturevalue(impl_name)
    model = mimi_models.synthetic_model()
    latents = mimi_models.synthetic_inputs(19)
    expected = mimi_models.synthetic_expected(latents)
    run = impl.mimi(model)
    try:
        ok, feats = run.process(latents)
        assert ok
        err = float(np.max(np.abs(feats - expected)))
        assert err <= 4e-6, err
        assert run.position == 19 * 16
        run.reset()  # framewise after reset
        parts = [run.process(latents[t:t + 1]) for t in range(19)]
        assert all(p[0] for p in parts)
        assert float(np.max(np.abs(np.concatenate([p[1] for p in parts]) - expected))) <= 4e-6
    finally:
        run.close()


@pytest.mark.parametrize("seed", [0, 1])
def test_oracle_vs_reference_random(oracle, reference, seed):
    model = mimi_models.random_model(seed)
    rng = np.random.default_rng(40 + seed)
    latents = rng.standard_normal((18, 32)).astype(np.float32)
    o, r = oracle.mimi(model), reference.mimi(model)
    try:
        ok_o, fo = o.process(latents)
        ok_r, fr = r.process(latents)
        assert ok_o and ok_r
        assert rel_err(fo, fr) < CHAIN_TOL, rel_err(fo, fr)
        # partitions of the same request give the same features (each implementation against itself)
        o.reset()
        parts = []
        for a, b in ((0, 1), (1, 8), (8, 18)):
            ok, f = o.process(latents[a:b])
            assert ok
            parts.append(f)
        assert np.array_equal(np.concatenate(parts), fo)
    finally:
        o.close()
        r.close()


@pytest.mark.parametrize("impl_name", ["oracle", "reference"])
def test_failure_contract(request, impl_name):
    impl = request.getfixturevalue(impl_name)
    model = mimi_models.random_model(3)
    run = impl.mimi(model)
    try:
        bad = np.zeros((2, 32), np.float32)
        bad[1, 5] = np.nan
        assert not run.process(bad)[0]
        assert run.position == 0  # rejected before processing starts
        assert run.process(np.zeros((1, 32), np.float32))[0]
    finally:
        run.close()

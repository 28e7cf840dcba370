"""The Mimi latent transformer on the GPU against the CPU oracle.

phonon_cuda_mimi_* run speech-mac's Mimi decoder transformer
(src/phonon_mimi.c:108-283) for a batch of request states, one latent frame
per state per step. Checked: the reference test's closed-form synthetic
model across the 250-key ring's wrap (tests/test_phonon_mimi.c:62-123, its
4e-6 absolute bound); random models against the oracle and the unmodified
reference build (chained bound 1e-3: the projections, attention and MLP sum
in another order than the reference's SGEMM calls); a batch of states equal
to each state run alone (bit for bit: every row's arithmetic is independent
of the batch); frame partitions of one request; the failure contracts."""
import numpy as np
import pytest

from phonon_b200 import runtime as rt

import mimi_models
from heads import rel_err

pytestmark = pytest.mark.gpu
CHAIN_TOL = 1e-3


def test_synthetic_closed_form(cuda_ok):
    model = mimi_models.synthetic_model()
    latents = mimi_models.synthetic_inputs(19)
    expected = mimi_models.synthetic_expected(latents)
    m = rt.Mimi(model, max_states=2, max_batch=2)
    try:
        s = m.alloc()
        feats = m.process(s, latents)
        err = float(np.max(np.abs(feats - expected)))
        print(f"mimi synthetic: max abs err {err:.2e} (bound 4e-6)")
        assert err <= 4e-6
        assert m.positions(s) == 19 * 16
        m.reset(s)
        frames = np.concatenate([m.process(s, latents[t:t + 1]) for t in range(19)])
        assert np.array_equal(frames, feats)
    finally:
        m.close()


@pytest.mark.parametrize("seed,tensor", [(0, False), (1, False), (0, True)])
def test_random_vs_oracle_and_reference(cuda_ok, oracle, reference, seed, tensor):
    """tensor: the four linears on the tensor cores (head_gemm_kernel, bf16
    weights x three bf16 slices), forced for this small batch."""
    model = mimi_models.random_model(seed)
    rng = np.random.default_rng(40 + seed)
    n, frames = 3, 18  # 288 positions: the ring wraps
    latents = rng.standard_normal((n, frames, 32)).astype(np.float32)
    m = rt.Mimi(model, max_states=4, max_batch=4)
    assert m.set_tensor_min(1 if tensor else 1 << 20), "tensor-core Mimi path unavailable"
    try:
        states = [m.alloc() for _ in range(n)]
        feats = np.zeros((n, frames * 16, 512), np.float32)
        for f in range(frames):
            out, status = m.step(states, latents[:, f])
            assert not status.any()
            feats[:, f * 16:(f + 1) * 16] = out
        worst_o = worst_r = 0.0
        for i in range(n):
            o = oracle.mimi(model)
            ok, fo = o.process(latents[i])
            o.close()
            assert ok
            worst_o = max(worst_o, rel_err(feats[i], fo))
        r = reference.mimi(model)
        ok, fr = r.process(latents[0])
        r.close()
        assert ok
        worst_r = rel_err(feats[0], fr)
        print(f"mimi seed {seed}{' tensor' if tensor else ''}: vs oracle {worst_o:.2e}, vs reference build {worst_r:.2e}")
        assert worst_o < CHAIN_TOL and worst_r < CHAIN_TOL
        # one state alone gives the same rows as in the batch
        s = m.alloc()
        alone = m.process(s, latents[1])
        assert np.array_equal(alone, feats[1])
    finally:
        m.close()


def test_failure_contracts(cuda_ok):
    model = mimi_models.random_model(3)
    m = rt.Mimi(model, max_states=2, max_batch=2)
    try:
        s = m.alloc()
        bad = np.zeros((2, 32), np.float32)
        bad[1, 5] = np.nan
        with pytest.raises(rt.CudaError) as e:
            m.process(s, bad)
        assert e.value.status == rt.NON_FINITE
        assert m.positions(s) == 0
        ok = m.process(s, np.zeros((1, 32), np.float32))
        assert np.isfinite(ok).all() and m.positions(s) == 16
        with pytest.raises(rt.CudaError):
            m.step([s, s], np.zeros((2, 32), np.float32))  # a state twice in one step
    finally:
        m.close()
    broken = mimi_models.random_model(3)
    broken["layers"][1]["scale2"] = broken["layers"][1]["scale2"].copy()
    broken["layers"][1]["scale2"][7] = 0x7FC0
    with pytest.raises(rt.CudaError) as e:
        rt.Mimi(broken)
    assert e.value.status == rt.NON_FINITE

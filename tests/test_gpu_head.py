"""The frame loop around the decode step on the GPU against the CPU oracle.

speech-mac's frame loop (src/speech.c:127-172) runs, per frame: the EOS
logit and one LSD Euler step of the flow head from the output-normed state
(src/phonon_sampler.c:280-402), the embedding of the new latent
(phonon_flow_embed_latent), the decode step, and phonon_flow_output_norm
(src/phonon_transformer.c:860-914). libphonon_cuda runs all of it on the
device (phonon_cuda_head_* and phonon_cuda_frame_step).

Bounds: the head chains six residual blocks of linears whose sums run in
another order than the reference's SGEMM, so its outputs are bounded like
the stack's final outputs, 1e-3 max relative error (heads.REL_TOL; the
oracle and the reference build differ by up to ~1.2e-4 on these heads). The
EOS logit is one dot product (bounded by 1e-5 of the sum of |w x|, the
scale of its rounding error, since the logit itself may be near zero); the
output norm is the transformer's LayerNorm and is bit-exact. In the frame
loop every frame is teacher-forced: the oracle starts from the device's
state, latent and K/V rows of that frame."""
import numpy as np
import pytest

from phonon_b200 import runtime as rt

import heads

pytestmark = pytest.mark.gpu
TOL = heads.REL_TOL
BF16 = 2  # oracle linear dtype


@pytest.fixture(scope="module")
def ctx(cuda_ok, weights12):
    c = rt.Context(weights12, max_streams=4, max_batch=16, pool_pages=64, kv_type=rt.KV_F32)
    yield c
    c.close()


def test_head_matches_reference_pin(ctx, pins):
    """The reference test's golden velocity (tests/test_phonon_sampler.c:148-197)."""
    p = pins["flow_head_synthetic"]
    h = rt.Head(ctx, heads.pinned_head())
    try:
        condition, state = heads.pinned_inputs()
        v = h.forward(condition[None], state[None], p["s"], p["t"])[0]
        err = float(np.max(np.abs(v - np.array(p["expected"], np.float32))))
        print(f"pinned head: max abs err {err:.2e} (bound {p['atol']})")
        assert err < p["atol"]
    finally:
        h.close()


@pytest.mark.parametrize("seed", [0, 1])
def test_head_batch_vs_oracle(ctx, oracle, reference, seed):
    head = heads.random_head(seed)
    h = rt.Head(ctx, head)
    rng = np.random.default_rng(200 + seed)
    n = 16
    cond = rng.standard_normal((n, 512)).astype(np.float32)
    state = rng.standard_normal((n, 32)).astype(np.float32)
    noise = rng.standard_normal((n, 32)).astype(np.float32)
    s, t = float(rng.uniform(0, 1)), float(rng.uniform(0, 1))
    try:
        v = h.forward(cond, state, s, t)
        y = h.lsd_one_step(cond, noise, 0.8)
        v2 = h.forward(cond[:3], state[:3], 0.25, 0.75)  # other times: embeddings recomputed
        # rows are independent of the batch they run in, bit for bit
        assert np.array_equal(h.forward(cond[5:6], state[5:6], s, t)[0], v[5])
        assert np.array_equal(h.lsd_one_step(cond[9:10], noise[9:10], 0.8)[0], y[9])
        worst = 0.0
        for i in range(n):
            ok, r = oracle.flow_head_forward(head, cond[i], state[i], s, t)
            assert ok
            worst = max(worst, heads.rel_err(v[i], r))
            ok, r = oracle.flow_lsd_one_step(head, cond[i], noise[i], 0.8)
            assert ok
            worst = max(worst, heads.rel_err(y[i], r))
        for i in range(3):
            ok, r = oracle.flow_head_forward(head, cond[i], state[i], 0.25, 0.75)
            assert ok
            worst = max(worst, heads.rel_err(v2[i], r))
        ref_worst = 0.0
        for i in range(4):  # the unmodified reference build as well
            ok, r = reference.flow_lsd_one_step(head, cond[i], noise[i], 0.8)
            assert ok
            ref_worst = max(ref_worst, heads.rel_err(y[i], r))
        print(f"head seed {seed}: vs oracle {worst:.2e}, vs reference build {ref_worst:.2e}")
        assert worst < TOL and ref_worst < TOL
    finally:
        h.close()


@pytest.fixture(scope="module")
def ctx64(cuda_ok, weights12):
    c = rt.Context(weights12, max_streams=4, max_batch=64, pool_pages=64, kv_type=rt.KV_F32)
    yield c
    c.close()


@pytest.mark.parametrize("n", [33, 64])
def test_head_tensor_path_vs_oracle(ctx64, oracle, n):
    """The tensor-core linears (bf16 weights x three bf16 slices of the fp32
    activations, head_gemm_kernel) on a partial and on full 32-stream tiles:
    against the oracle at the head's bound, and against the GEMV path."""
    head = heads.random_head(11)
    h = rt.Head(ctx64, head)
    rng = np.random.default_rng(300 + n)
    cond = rng.standard_normal((n, 512)).astype(np.float32)
    state = rng.standard_normal((n, 32)).astype(np.float32)
    noise = rng.standard_normal((n, 32)).astype(np.float32)
    try:
        assert h.set_tensor_min(1), "tensor-core head path unavailable"
        v = h.forward(cond, state, 0.3, 0.9)
        y = h.lsd_one_step(cond, noise, 0.8)
        h.set_tensor_min(1 << 30)
        v_gemv = h.forward(cond, state, 0.3, 0.9)
        worst = 0.0
        for i in range(n):
            ok, r = oracle.flow_head_forward(head, cond[i], state[i], 0.3, 0.9)
            assert ok
            worst = max(worst, heads.rel_err(v[i], r))
            ok, r = oracle.flow_lsd_one_step(head, cond[i], noise[i], 0.8)
            assert ok
            worst = max(worst, heads.rel_err(y[i], r))
        between = max(heads.rel_err(v[i], v_gemv[i]) for i in range(n))
        print(f"tensor head, {n} rows: vs oracle {worst:.2e}, vs GEMV path {between:.2e}")
        assert worst < TOL and between < TOL
    finally:
        h.close()


def test_head_failure_contracts(ctx):
    """The reference's checks (src/phonon_sampler.c:307-393): non-finite
    state or noise rows, non-finite times, temperature <= 0, non-finite
    weights. A failed call writes nothing and leaves the head usable."""
    head = heads.random_head(5)
    h = rt.Head(ctx, head)
    try:
        cond = np.ones((2, 512), np.float32)
        state = np.zeros((2, 32), np.float32)
        good = h.forward(cond, state, 0.0, 1.0)
        bad = state.copy()
        bad[1, 3] = np.nan
        for call in (lambda: h.forward(cond, bad, 0.0, 1.0), lambda: h.forward(cond, state, float("inf"), 1.0),
                     lambda: h.lsd_one_step(cond, bad, 1.0)):
            with pytest.raises(rt.CudaError) as e:
                call()
            assert e.value.status == rt.NON_FINITE
        with pytest.raises(rt.CudaError) as e:
            h.lsd_one_step(cond, state, 0.0)
        assert e.value.status == rt.INVALID
        assert np.array_equal(h.forward(cond, state, 0.0, 1.0), good)
    finally:
        h.close()
    broken = heads.random_head(5)
    broken["block_norm_w"][2] = broken["block_norm_w"][2].copy()
    broken["block_norm_w"][2][9] = 0x7FC0  # a NaN gain
    with pytest.raises(rt.CudaError) as e:
        rt.Head(ctx, broken)
    assert e.value.status == rt.NON_FINITE


def test_eos_logit_and_output_norm(ctx, oracle):
    import torch
    fr = heads.random_frame(3)
    h = rt.Head(ctx, heads.random_head(3), fr)
    rng = np.random.default_rng(33)
    try:
        state = rng.standard_normal((16, 512)).astype(np.float32)
        logit = h.eos_logit(state)
        w_eos, b_eos = heads.widen(fr["eos"][0]).reshape(512), heads.widen(fr["eos"][1])
        for i in range(16):
            ok, r = oracle.linear(BF16, fr["eos"][0], 1, 512, state[i], bias=b_eos)
            assert ok
            bound = 1e-5 * float(np.sum(np.abs(w_eos * state[i]))) + 1e-7
            assert abs(float(logit[i]) - float(r[0])) <= bound, (i, logit[i], r[0])
        x = torch.tensor(state, device="cuda")
        y = torch.empty_like(x)
        h.output_norm_device(16, x.data_ptr(), y.data_ptr())
        out = y.cpu().numpy()
        w, b = heads.widen(fr["out_norm"][0]), heads.widen(fr["out_norm"][1])
        for i in range(16):
            ok, r = oracle.layer_norm(state[i], w, b, 1e-5)
            assert ok and np.array_equal(out[i], r), i
        bad = state.copy()
        bad[4, 100] = np.inf
        with pytest.raises(rt.CudaError) as e:
            h.eos_logit(bad)
        assert e.value.status == rt.NON_FINITE
    finally:
        h.close()


@pytest.mark.parametrize("n", [1, 8, 40])
def test_frame_loop_vs_oracle(cuda_ok, oracle, weights12, n):
    """Frames of n streams through phonon_cuda_frame_step (n = 1 takes the
    cluster step, n = 8 the persistent step and the head's GEMV linears,
    n = 40 the tensor-core projections and head linears), each frame checked against the
    oracle from the device's state and K/V rows: the EOS logit, the latent,
    and the new state (embedding, 12-layer step, output norm)."""
    import torch
    lens = [40 + 13 * i for i in range(n)]
    pages = sum((ln + 4) // 16 + 1 for ln in lens) + 16
    ctx = rt.Context(weights12, max_streams=n + 2, max_batch=n, pool_pages=pages, kv_type=rt.KV_F32)
    head, fr = heads.random_head(7), heads.random_frame(7)
    h = rt.Head(ctx, head, fr)
    om = oracle.model(weights12)
    rng = np.random.default_rng(70 + n)
    w_on, b_on = heads.widen(fr["out_norm"][0]), heads.widen(fr["out_norm"][1])
    b_eos = heads.widen(fr["eos"][1])
    w_eos = heads.widen(fr["eos"][0]).reshape(512)
    try:
        streams = [ctx.stream_alloc(1024) for _ in range(n)]
        for i, s in enumerate(streams):
            ctx.fill_synthetic(s, lens[i], 500 + i)
        state0 = np.stack([oracle.layer_norm(rng.standard_normal(512).astype(np.float32), w_on, b_on)[1]
                           for _ in range(n)])
        cond = (0.5 * rng.standard_normal((n, 512))).astype(np.float32)
        state_dev = torch.tensor(state0, device="cuda")
        cond_dev = torch.tensor(cond, device="cuda")
        worst = {"latent": 0.0, "logit": 0.0, "state": 0.0}
        for f in range(4):
            before = state_dev.cpu().numpy().copy()
            raw = rng.standard_normal((n, 32)).astype(np.float32)
            pos = [ln + f for ln in lens]
            logit, lat, status = h.frame_step(streams, pos, state_dev.data_ptr(), cond_dev.data_ptr(), raw, 0.8)
            assert (status == rt.OK).all(), status
            after = state_dev.cpu().numpy()
            for i in range(n):
                ok, r_lat = oracle.flow_lsd_one_step(head, before[i], raw[i], 0.8)
                assert ok
                worst["latent"] = max(worst["latent"], heads.rel_err(lat[i], r_lat))
                ok, r_lg = oracle.linear(BF16, fr["eos"][0], 1, 512, before[i], bias=b_eos)
                assert ok
                scale = float(np.sum(np.abs(w_eos * before[i])))  # the dot product's own magnitude
                worst["logit"] = max(worst["logit"], abs(float(logit[i]) - float(r_lg[0])) / scale)
                ok, e = oracle.linear(BF16, fr["embed"], 512, 32, lat[i])
                assert ok
                x = (e + cond[i]).astype(np.float32)
                k, v = ctx.kv_read(streams[i], 0, pos[i])
                cache = om.new_stream(pos[i] + 1)
                try:
                    om.load_kv(cache, k, v)
                    cache.length = pos[i]
                    ok, y, _ = om.step(cache, pos[i], x)
                    assert ok
                finally:
                    om.free_stream(cache)
                ok, r_state = oracle.layer_norm(y, w_on, b_on)
                assert ok
                worst["state"] = max(worst["state"], heads.rel_err(after[i], r_state))
        for i, s in enumerate(streams):
            assert ctx.length(s) == lens[i] + 4
        print(f"frame loop, {n} streams x 4 frames: " + ", ".join(f"{k} {v:.2e}" for k, v in worst.items()))
        assert worst["latent"] < TOL and worst["state"] < TOL and worst["logit"] < 1e-5, worst
    finally:
        h.close()
        ctx.close()

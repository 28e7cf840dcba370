"""Two-lane decode steps (a large batch as two concurrent half batches).

Every projection is exact per stream row, so the first layer's K/V rows,
appended before any attention, are the same bit for bit on two lanes as on
one. A two-lane step cuts attention into fewer, longer splits (each half's
attention leaves SMs to the other half), so later layers differ from a
one-lane step only in the order attention partials are merged. The
comparison is teacher-forced: after every step the two-lane context gets the
one-lane context's appended K/V rows (bf16 K/V would otherwise let 1-ulp
differences flip roundings and compound over steps), and the outputs of each
step then agree within the final-output tolerance of the reference's tests
(1e-3 max relative error; measured ~7e-5 after 12 layers; a wrong row or
lane mix-up shows as O(1)). Covered with the tensor-core projections and with the GEMV ones,
bf16 and fp32 K/V, across page boundaries."""
import numpy as np
import pytest

from phonon_b200 import runtime as rt

pytestmark = pytest.mark.gpu
NEVER = 1 << 20


@pytest.mark.parametrize("kv_type,tensor_min", [(rt.KV_BF16, 32), (rt.KV_F32, 32), (rt.KV_BF16, NEVER)])
def test_two_lanes_equal_one(cuda_ok, weights12, kv_type, tensor_min):
    R = 131
    kw = dict(max_streams=R + 4, max_batch=R, pool_pages=R * 12, kv_type=kv_type)
    two, one = rt.Context(weights12, **kw), rt.Context(weights12, **kw)
    try:
        two.set_batch_paths(NEVER, rt.FUSED_MAX_BATCH, tensor_min, 96)
        one.set_batch_paths(NEVER, rt.FUSED_MAX_BATCH, tensor_min, NEVER)
        rng = np.random.default_rng(3)
        lengths = rng.integers(1, 150, size=R)
        st, so = [two.stream_alloc(200) for _ in range(R)], [one.stream_alloc(200) for _ in range(R)]
        for i in range(R):
            two.fill_synthetic(st[i], int(lengths[i]), 40 + i)
            one.fill_synthetic(so[i], int(lengths[i]), 40 + i)
        for step in range(8):
            pos = [int(lengths[i]) + step for i in range(R)]
            x = rng.standard_normal((R, 512)).astype(np.float32)
            y2, y1 = two.step(st, pos, x), one.step(so, pos, x)
            assert rt.rel_err(y2, y1) < 1e-3, (step, rt.rel_err(y2, y1))
            for i in range(R):
                k2, v2 = two.kv_read(st[i], pos[i], 1, layer_begin=0, layer_count=1)
                k1, v1 = one.kv_read(so[i], pos[i], 1)
                assert np.array_equal(k2, k1[:1]) and np.array_equal(v2, v1[:1]), (step, i)
                two.kv_write(st[i], pos[i], k1, v1)  # teacher forcing: same caches for the next step
    finally:
        two.close()
        one.close()

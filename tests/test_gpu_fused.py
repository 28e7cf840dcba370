"""Whole-step persistent launch (batches up to PHONON_CUDA_FUSED_MAX_BATCH).

The persistent kernel repeats the per-lane arithmetic of the per-stage GEMV,
attention and split-merge kernels, so for the same batch the two paths agree
bit for bit: the step outputs and every K/V row the step appends. Two
contexts with the same weights and the same synthetic caches run the same
steps, one through each path (the per-stage one with the tensor-core
projections switched off). Positions cross page boundaries, so page-table
updates happen inside the persistent launch. Parity of the persistent path
with the CPU oracle is covered by test_gpu_step (its batches are small
enough to take this path)."""
import numpy as np
import pytest

from phonon_b200 import runtime as rt
from phonon_b200 import synth

pytestmark = pytest.mark.gpu
NO_TENSOR = 1 << 20


def _pair(weights, kv_type):
    kw = dict(max_streams=72, max_batch=64, pool_pages=2048, kv_type=kv_type)
    fused = rt.Context(weights, **kw)
    fused.set_batch_paths(1, rt.FUSED_MAX_BATCH, NO_TENSOR)
    staged = rt.Context(weights, **kw)
    staged.set_batch_paths(rt.FUSED_MAX_BATCH + 1, rt.FUSED_MAX_BATCH, NO_TENSOR)
    for c in (fused, staged):  # single-stream steps too: no cluster path
        c.set_cluster_step(0)
    return fused, staged


@pytest.mark.parametrize("kv_type,batches", [(rt.KV_BF16, (1, 5, 8, 13, 64)), (rt.KV_F32, (1, 8, 13, 40))])
def test_fused_equals_staged_bitwise(cuda_ok, weights12, kv_type, batches):
    fused, staged = _pair(weights12, kv_type)
    rng = np.random.default_rng(7)
    try:
        for R in batches:
            lengths = rng.integers(1, 300, size=R)
            sf = [fused.stream_alloc(400) for _ in range(R)]
            ss = [staged.stream_alloc(400) for _ in range(R)]
            for i in range(R):
                fused.fill_synthetic(sf[i], int(lengths[i]), 1000 + i)
                staged.fill_synthetic(ss[i], int(lengths[i]), 1000 + i)
            for step in range(18):
                pos = [int(lengths[i]) + step for i in range(R)]
                x = rng.standard_normal((R, 512)).astype(np.float32)
                l0 = fused.launch_count()
                yf = fused.step(sf, pos, x)
                launches = fused.launch_count() - l0
                ys = staged.step(ss, pos, x)
                assert launches == 1, f"R={R}: {launches} launches for one fused step"
                assert np.array_equal(yf, ys), (R, step, float(np.max(np.abs(yf - ys))))
            for i in range(R):
                first = int(lengths[i])
                kf, vf = fused.kv_read(sf[i], first, 18)
                ks, vs = staged.kv_read(ss[i], first, 18)
                assert np.array_equal(kf, ks) and np.array_equal(vf, vs), (R, i)
                assert len(fused.pages(sf[i])) == len(staged.pages(ss[i])) > 0
            for s in sf:
                fused.stream_free(s)
            for s in ss:
                staged.stream_free(s)
    finally:
        fused.close()
        staged.close()


def test_fused_step_device_and_reuse(cuda_ok, weights12):
    """Device-buffer steps through the persistent path, back to back, with the
    output buffer reused as the next input (as a decode loop does)."""
    import torch
    fused, staged = _pair(weights12, rt.KV_BF16)
    try:
        R = 12
        sf = [fused.stream_alloc(256) for _ in range(R)]
        ss = [staged.stream_alloc(256) for _ in range(R)]
        for i in range(R):
            fused.fill_synthetic(sf[i], 30 + 7 * i, 5 + i)
            staged.fill_synthetic(ss[i], 30 + 7 * i, 5 + i)
        g = synth.Generator(3)
        x0 = g.normal(R * 512).reshape(R, 512).astype(np.float32)
        buf = [torch.tensor(x0, device="cuda"), torch.empty(R, 512, device="cuda")]
        xs = x0
        for step in range(10):
            pos = [30 + 7 * i + step for i in range(R)]
            fused.step_device(sf, pos, buf[step & 1].data_ptr(), buf[(step + 1) & 1].data_ptr())
            assert not fused.sync(R).any()
            xs = staged.step(ss, pos, xs)
        assert np.array_equal(buf[0].cpu().numpy(), xs)
    finally:
        fused.close()
        staged.close()

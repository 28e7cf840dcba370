"""Single-stream decode steps on one 16-CTA cluster (step_cluster_kernel).

The cluster path runs every layer of a one-stream step in one launch. Its
LayerNorm, projections, RoPE and K/V appends repeat the arithmetic of a
per-stage path, so the first layer's appended K/V rows (which depend on
nothing but the step input and the weights) equal that path's bit for bit:
the GEMV path's when every projection runs on the CUDA cores (weights with
per-block scales), the tensor-core path's when the projections run on the
tensor cores (one scale per row, the synthetic configs);
the attention merges its partial sums in another order, so everything after
the first attention agrees within rounding (fp32 K/V: 1e-3; bf16 K/V: 1e-2,
a rounding-level difference can flip a bf16 rounding). Against the CPU oracle the
chained output is bounded by 1e-3 (configs[0] in test_gpu_step also runs on
this path). Positions cover one page (the second CTA of every head idle), page
boundaries, more pages per CTA than its 8-slot page ring, and long contexts."""
import numpy as np
import pytest

from phonon_b200 import runtime as rt
from phonon_b200 import synth

pytestmark = pytest.mark.gpu
FINAL_TOL = 1e-3


def _pair(weights, kv_type):
    kw = dict(max_streams=8, max_batch=4, pool_pages=1024, kv_type=kv_type)
    cl = rt.Context(weights, **kw)
    staged = rt.Context(weights, **kw)
    form = cl.set_cluster_step(rt.MAX_POSITIONS)
    assert form, "16-CTA cluster step unavailable on this device"
    staged.set_cluster_step(0)
    if form == 2:  # the per-stage path with the same (tensor-core) q/k/v arithmetic
        staged.set_batch_paths(tensor_min_batch=1)
    return cl, staged, form


@pytest.fixture(scope="module")
def weights12_blocks(weights12):
    from phonon_b200 import synth as s
    return s.per_block_scales(weights12, 5)


@pytest.mark.parametrize("scales", ["row", "block"])
@pytest.mark.parametrize("kv_type", [rt.KV_F32, rt.KV_BF16])
@pytest.mark.parametrize("length", [0, 5, 14, 127, 290, 1500])
def test_cluster_equals_staged_path(cuda_ok, weights12, weights12_blocks, kv_type, length, scales):
    cl, staged, form = _pair(weights12 if scales == "row" else weights12_blocks, kv_type)
    assert form == (2 if scales == "row" else 1)
    try:
        a, b = cl.stream_alloc(2048), staged.stream_alloc(2048)
        if length:
            cl.fill_synthetic(a, length, 99)
            staged.fill_synthetic(b, length, 99)
        g = synth.Generator(1234 + length)
        worst = 0.0
        for step in range(20):
            pos = length + step
            x = g.normal(512)[None]
            l0 = cl.launch_count()
            ya = cl.step([a], [pos], x)
            assert cl.launch_count() - l0 == 1
            yb = staged.step([b], [pos], x)
            worst = max(worst, rt.rel_err(ya[0], yb[0]))
        ka, va = cl.kv_read(a, length, 20)
        kb, vb = staged.kv_read(b, length, 20)
        assert np.array_equal(ka[0], kb[0]) and np.array_equal(va[0], vb[0])  # layer 0: bit for bit
        # bf16 K/V: a rounding-level difference before the bf16 rounding can
        # flip it (2^-8 relative), as in test_gpu_step's bf16 test (measured
        # up to 1.16e-2 on the tensor-core form)
        tol = FINAL_TOL if kv_type == rt.KV_F32 else 2e-2
        assert rt.rel_err(ka.ravel(), kb.ravel()) < tol and rt.rel_err(va.ravel(), vb.ravel()) < tol
        assert cl.length(a) == staged.length(b) == length + 20
        assert list(cl.pages(a)) == list(staged.pages(b))
        assert worst < tol, worst
    finally:
        cl.close()
        staged.close()


def test_cluster_chain_vs_oracle(cuda_ok, oracle, weights12):
    """Positions 0..47 chained through the cluster path against the oracle
    (first steps on one page, then page boundaries at 16 and 32)."""
    ctx = rt.Context(weights12, max_streams=2, max_batch=2, pool_pages=64)
    assert ctx.set_cluster_step(rt.MAX_POSITIONS)
    om = oracle.model(weights12)
    oc = om.new_stream(64)
    s = ctx.stream_alloc(64)
    g = synth.stream_generator(0, 3)
    worst = 0.0
    try:
        for pos in range(48):
            x = g.normal(512)
            y = ctx.step([s], [pos], x[None])[0]
            ok, ref, _ = om.step(oc, pos, x)
            assert ok
            worst = max(worst, rt.rel_err(y, ref))
        k, v = ctx.kv_read(s, 0, 48)
        ko = np.stack([[om.kv(oc, l, p)[0] for p in range(48)] for l in range(12)])
        assert rt.rel_err(k.ravel(), ko.ravel()) < FINAL_TOL  # the oracle sums its linears in another order
    finally:
        om.free_stream(oc)
        ctx.close()
    assert worst < FINAL_TOL, worst


def test_cluster_long_prefix_vs_oracle(cuda_ok, oracle, weights12):
    """A 300-position prefix (10 pages per CTA: the page ring wraps within
    a layer), then decode steps, against the oracle."""
    ctx = rt.Context(weights12, max_streams=2, max_batch=2, pool_pages=64)
    assert ctx.set_cluster_step(rt.MAX_POSITIONS)
    om = oracle.model(weights12)
    oc = om.new_stream(320)
    s = ctx.stream_alloc(320)
    g = synth.stream_generator(4, 0)
    prefix = np.stack([g.normal(512) for _ in range(300)])
    worst = 0.0
    try:
        ctx.append(s, prefix)
        for pos in range(300):
            om.step(oc, pos, prefix[pos])
        for pos in range(300, 310):
            x = g.normal(512)
            y = ctx.step([s], [pos], x[None])[0]
            ok, ref, _ = om.step(oc, pos, x)
            assert ok
            worst = max(worst, rt.rel_err(y, ref))
    finally:
        om.free_stream(oc)
        ctx.close()
    assert worst < FINAL_TOL, worst


def test_cluster_nonfinite_input(cuda_ok, weights12):
    """A non-finite input fails the step: status NON_FINITE, nothing committed,
    the output row left as it was; the stream steps on afterwards."""
    ctx = rt.Context(weights12, max_streams=2, max_batch=2, pool_pages=16)
    assert ctx.set_cluster_step(rt.MAX_POSITIONS)
    s = ctx.stream_alloc(32)
    try:
        x = synth.Generator(5).normal(512)[None].copy()
        x[0, 7] = np.nan
        out = np.full((1, 512), 3.0, np.float32)
        _, st = ctx.step([s], [0], x, raise_on_status=False, out=out)
        assert list(st) == [rt.NON_FINITE] and ctx.length(s) == 0 and np.all(out == 3.0)
        x[0, 7] = 0.5
        y = ctx.step([s], [0], x)
        assert np.all(np.isfinite(y)) and ctx.length(s) == 1
    finally:
        ctx.close()


def test_cluster_default_window(cuda_ok, weights12):
    """By default one stream's step runs on the cluster below 1152 positions
    (fp32 K/V) and per stage from there on, where the attention over all SMs
    is faster than over the cluster's 16."""
    ctx = rt.Context(weights12, max_streams=2, max_batch=2, pool_pages=160, kv_type=rt.KV_F32)
    try:
        s = ctx.stream_alloc(2048)
        ctx.fill_synthetic(s, 1151, 3)
        x = synth.Generator(9).normal(512)[None]
        l0 = ctx.launch_count()
        ctx.step([s], [1151], x)
        assert ctx.launch_count() - l0 == 1  # one cluster launch
        l0 = ctx.launch_count()
        ctx.step([s], [1152], x)
        assert ctx.launch_count() - l0 > 1  # the per-stage launches
    finally:
        ctx.close()

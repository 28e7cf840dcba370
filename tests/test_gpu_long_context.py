"""Long contexts on every decode path, layer by layer (fp32 K/V).

Five streams attend over 513, 1025, 1537, 4096 and 4352 keys (the reference
test's attention pins at 513/1025/1537 keys, tests/test_speech.c:120-169,
and configs[4]'s long-form contexts up to 4352). The same steps run on each
path a decode step can take: the per-stage GEMVs, the per-stage tcgen05
projections, the persistent whole-step kernel (one batch of five) and the
16-CTA cluster kernel (five single-stream steps). Every layer of two steps is
teacher-forced against the oracle (tests/parity.py) and bounded at 1e-4; on
the cluster path (the default for one stream) the unmodified reference build
(oracle/_ref) is checked directly as well."""
import numpy as np
import pytest

from phonon_b200 import runtime as rt
from phonon_b200 import synth

import parity

pytestmark = pytest.mark.gpu
NEVER = 1 << 20
POSITIONS = [512, 1024, 1536, 4095, 4351]  # keys attended: position + 1
STEPS = 2
# (fused window, tensor-core minimum, cluster step)
PATHS = {
    "gemv": ((NEVER, rt.FUSED_MAX_BATCH, NEVER), False),
    "tensor": ((NEVER, rt.FUSED_MAX_BATCH, 1), False),
    "persistent": ((1, rt.FUSED_MAX_BATCH, NEVER), False),
    "cluster": (None, True),
}


@pytest.fixture(scope="module")
def long_ctx(cuda_ok, weights12):
    pages = len(POSITIONS) * ((max(POSITIONS) + STEPS) // 16 + 2) + 16
    c = rt.Context(weights12, max_streams=8, max_batch=8, pool_pages=pages, kv_type=rt.KV_F32)
    yield c
    c.close()


def _run(ctx, path):
    paths, cluster = PATHS[path]
    if paths:
        ctx.set_batch_paths(*paths)
    ctx.set_cluster_step(rt.MAX_POSITIONS if cluster else 0)
    n = len(POSITIONS)
    trace = parity.Trace(ctx, n)
    streams = [ctx.stream_alloc(max(POSITIONS) + STEPS + 16) for _ in range(n)]
    try:
        for i, (s, p) in enumerate(zip(streams, POSITIONS)):
            ctx.fill_synthetic(s, p, 77 + i)
        g = synth.Generator(4352)
        xs, traces = [], []
        for t in range(STEPS):
            x = g.normal(n * 512).reshape(n, 512)
            pos = [p + t for p in POSITIONS]
            if cluster:  # one stream per step: each step's trace holds one row
                tr = np.zeros((ctx.n_layers, n, 512), np.float32)
                for i in range(n):
                    y = ctx.step([streams[i]], [pos[i]], x[i:i + 1])
                    tr[:, i] = trace.read(1)[:, 0]
                    assert np.array_equal(tr[-1, i], y[0])
            else:
                y = ctx.step(streams, pos, x)
                tr = trace.read(n)
                assert np.array_equal(tr[-1], y)
            xs.append(x)
            traces.append(tr)
        return streams, xs, traces
    except Exception:
        for s in streams:
            ctx.stream_free(s)
        raise
    finally:
        trace.close()
        ctx.set_batch_paths()
        ctx.set_cluster_step(rt.MAX_POSITIONS)


@pytest.mark.parametrize("path", list(PATHS))
def test_long_context_per_layer(long_ctx, oracle, weights12, path):
    if path == "cluster":
        assert long_ctx.set_cluster_step(rt.MAX_POSITIONS), "cluster step unavailable"
    streams, xs, traces = _run(long_ctx, path)
    try:
        om = oracle.model(weights12)
        stats = parity.Stats()
        for i, p in enumerate(POSITIONS):
            parity.check_stream_oracle(long_ctx, om, streams[i], [p + t for t in range(STEPS)],
                                       [x[i] for x in xs], traces, i, stats, kv_bf16=False,
                                       label=f"{path} keys {p + 1}")
        print(f"{path}: oracle {stats}")
        assert stats.rel < parity.PER_LAYER_TOL, str(stats)
        assert stats.kv_rel < parity.PER_LAYER_TOL, str(stats)  # fp32 rows: equal up to summation order
    finally:
        for s in streams:
            long_ctx.stream_free(s)


def test_long_context_cluster_vs_reference_build(long_ctx, reference, weights12):
    """The default single-stream path against the unmodified reference C
    (oracle/_ref: src/phonon_transformer.c's phonon_flow_layer_step over the
    reference's contiguous PhononKvCache holding the device's K/V rows)."""
    assert long_ctx.set_cluster_step(rt.MAX_POSITIONS), "cluster step unavailable"
    streams, xs, traces = _run(long_ctx, "cluster")
    try:
        rm = reference.model(weights12, prepare=True)
        stats = parity.Stats()
        for i, p in enumerate(POSITIONS):
            parity.check_stream_reference(long_ctx, rm, streams[i], [p + t for t in range(STEPS)],
                                          [x[i] for x in xs], traces, i, stats, label=f"keys {p + 1}")
        print(f"cluster vs reference build: {stats}")
        assert stats.rel < parity.PER_LAYER_TOL, str(stats)
    finally:
        for s in streams:
            long_ctx.stream_free(s)

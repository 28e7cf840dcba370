"""The tcgen05 int8 tensor-core path of the batched step.

The projections of a batch of >= 32 streams run as int8 MMAs over
digit-sliced activations: the integer accumulation is checked bit for bit
against a CPU integer product, and the recombined fp32 results against the
CUDA-core GEMV path and the CPU oracle."""
import numpy as np
import pytest

from phonon_b200 import runtime as rt
from phonon_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k", [(128, 128, 128), (1536, 256, 512), (512, 2048, 2048),
                                   (2048, 384, 512), (130, 70, 256)])
def test_i8_gemm_bit_exact(cuda_ok, m, n, k):
    rng = np.random.default_rng(m * 7 + n)
    a = rng.integers(-127, 128, (m, k)).astype(np.int8)
    b = rng.integers(-64, 65, (n, k)).astype(np.int8)
    d = rt.i8_gemm(a, b)
    assert np.array_equal(d.astype(np.int64), a.astype(np.int64) @ b.astype(np.int64).T)


def test_i8_gemm_extremes(cuda_ok):
    a = np.full((128, 2048), -127, np.int8)
    b = np.full((128, 2048), -64, np.int8)
    assert np.all(rt.i8_gemm(a, b) == 2048 * 127 * 64)


@pytest.fixture(scope="module")
def ctx12t(cuda_ok, weights12):
    c = rt.Context(weights12, max_streams=96, max_batch=64, pool_pages=2048)
    yield c
    c.close()


def test_tensor_path_matches_gemv_path(ctx12t):
    n = 48
    streams = [ctx12t.stream_alloc(700) for _ in range(n)]
    lens = [int(x) for x in np.random.default_rng(4).integers(16, 600, n)]
    x = synth.Generator(12).normal(n * 512).reshape(n, 512)

    def fresh():
        for s, ln in zip(streams, lens):
            ctx12t.stream_reset(s)
            ctx12t.fill_synthetic(s, ln, 77 + s)

    fresh()
    y_tensor = ctx12t.step(streams, lens, x)          # B = 48: tcgen05 projections
    fresh()
    y_gemv = np.stack([ctx12t.step([s], [ln], x[i:i + 1])[0] for i, (s, ln) in
                       enumerate(zip(streams, lens))])  # B = 1: CUDA-core GEMV
    for s in streams:
        ctx12t.stream_free(s)
    worst = max(rt.rel_err(a, b) for a, b in zip(y_tensor, y_gemv))
    print(f"tensor vs GEMV path, 12 layers: max rel err {worst:.2e}")
    assert worst < 1e-3


def test_tensor_path_vs_oracle(ctx12t, oracle, weights12):
    om = oracle.model(weights12)
    n = 40
    streams = [ctx12t.stream_alloc(64) for _ in range(n)]
    caches = [om.new_stream(64) for _ in range(n)]
    gens = [synth.stream_generator(6, i) for i in range(n)]
    worst = 0.0
    for pos in range(20):
        xs = np.stack([g.normal(512) for g in gens])
        ys = ctx12t.step(streams, [pos] * n, xs)
        for i in range(n):
            ok, ref, _ = om.step(caches[i], pos, xs[i])
            assert ok
            worst = max(worst, rt.rel_err(ys[i], ref))
    for s in streams:
        ctx12t.stream_free(s)
    for c in caches:
        om.free_stream(c)
    print(f"tensor path vs oracle, 40 streams x 20 steps: max rel err {worst:.2e}")
    assert worst < 1e-3, worst


def test_per_block_scales_on_the_tensor_cores(cuda_ok, oracle, weights12):
    """Per-block-scale Q8_0 linears take the three-digit-plane tcgen05 path
    (a batch of 40 streams): every layer teacher-forced against the oracle,
    which applies each block's scale itself, within the per-layer bound; and
    the step against the CUDA-core GEMV path of the same weights."""
    import parity
    weights = synth.per_block_scales(weights12, 5)
    n = 40
    ctx = rt.Context(weights, max_streams=n + 4, max_batch=n, pool_pages=1024, kv_type=rt.KV_F32)
    gemv = rt.Context(weights, max_streams=n + 4, max_batch=n, pool_pages=1024, kv_type=rt.KV_F32)
    gemv.set_batch_paths(rt.FUSED_MAX_BATCH + 1, rt.FUSED_MAX_BATCH, 1 << 20)
    trace = parity.Trace(ctx, n)
    try:
        lens = [20 + 7 * i for i in range(n)]
        ss = [ctx.stream_alloc(600) for _ in range(n)]
        sg = [gemv.stream_alloc(600) for _ in range(n)]
        for i in range(n):
            ctx.fill_synthetic(ss[i], lens[i], 300 + i)
            gemv.fill_synthetic(sg[i], lens[i], 300 + i)
        g = synth.Generator(17)
        xs, traces, worst_gemv = [], [], 0.0
        for t in range(2):
            x = g.normal(n * 512).reshape(n, 512)
            pos = [ln + t for ln in lens]
            l0 = ctx.launch_count()
            y = ctx.step(ss, pos, x)
            launches = ctx.launch_count() - l0
            traces.append(trace.read(n))
            xs.append(x)
            l0 = gemv.launch_count()
            yg = gemv.step(sg, pos, x)
            # the tensor path runs nine launches per layer (digit slicing + GEMMs), the GEMV path fewer
            assert launches > gemv.launch_count() - l0, (launches, gemv.launch_count() - l0)
            worst_gemv = max(worst_gemv, rt.rel_err(y, yg))
        om = oracle.model(weights)
        stats = parity.Stats()
        for i in (0, 13, 27, 39):
            parity.check_stream_oracle(ctx, om, ss[i], [lens[i], lens[i] + 1], [x[i] for x in xs], traces, i, stats,
                                       kv_bf16=False, label=f"stream {i}")
        print(f"per-block scales, tensor path: {stats}; vs GEMV path {worst_gemv:.2e}")
        assert stats.rel < parity.PER_LAYER_TOL, str(stats)
        assert worst_gemv < 1e-3
    finally:
        trace.close()
        ctx.close()
        gemv.close()

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

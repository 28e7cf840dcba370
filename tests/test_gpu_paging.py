"""KV page pool: page-table contents against a CPU restatement of the
allocator, free-list churn, exhaustion and rollback, request isolation."""
import numpy as np
import pytest

from phonon_b200 import runtime as rt
from phonon_b200 import synth

pytestmark = pytest.mark.gpu


class PoolModel:
    """CPU restatement of the page allocator: a LIFO free list seeded with
    pages 0..P-1 (page 0 on top); streams take pages in position order and
    return them in reverse on reset/free."""

    def __init__(self, n):
        self.free = list(range(n - 1, -1, -1))
        self.pages = {}

    def ensure(self, s, n):
        p = self.pages.setdefault(s, [])
        while len(p) < n:
            p.append(self.free.pop())

    def release(self, s):
        for page in reversed(self.pages.get(s, [])):
            self.free.append(page)
        self.pages[s] = []


@pytest.fixture(scope="module")
def small_ctx(cuda_ok):
    w = synth.flow_weights(2, seed=4)
    c = rt.Context(w, max_streams=8, max_batch=8, pool_pages=24)
    yield c
    c.close()


def test_page_table_matches_allocator_model(small_ctx):
    model = PoolModel(24)
    streams = [small_ctx.stream_alloc(256) for _ in range(3)]
    g = synth.Generator(3)
    pos = [0, 0, 0]
    rng = np.random.default_rng(0)
    for it in range(60):
        act = sorted(set(rng.integers(0, 3, 2).tolist()))
        xs = g.normal(len(act) * 512).reshape(len(act), 512)
        small_ctx.step([streams[i] for i in act], [pos[i] for i in act], xs)
        for i in act:
            model.ensure(i, pos[i] // 16 + 1)
            pos[i] += 1
        if it == 30:
            small_ctx.stream_reset(streams[1])
            model.release(1)
            pos[1] = 0
        for i in range(3):
            assert list(small_ctx.pages(streams[i])) == model.pages.get(i, [])
    assert small_ctx.free_pages() == len(model.free)
    for s in streams:
        small_ctx.stream_free(s)
    assert small_ctx.free_pages() == 24


def test_kv_rows_round_trip_bit_exact(small_ctx):
    s = small_ctx.stream_alloc(100)
    g = synth.Generator(5)
    keys = g.normal(2 * 37 * 512).reshape(2, 37, 512)
    vals = g.normal(2 * 37 * 512).reshape(2, 37, 512)
    small_ctx.kv_write(s, 3, keys, vals)
    k, v = small_ctx.kv_read(s, 3, 37)
    assert np.array_equal(k, keys) and np.array_equal(v, vals)
    k, _ = small_ctx.kv_read(s, 90, 10)  # pages never allocated read as zero
    assert not k.any()
    bad = keys.copy()
    bad[1, 5, 7] = np.inf
    with pytest.raises(rt.CudaError) as e:
        small_ctx.kv_write(s, 3, bad, vals)
    assert e.value.status == rt.NON_FINITE
    small_ctx.stream_free(s)


def test_pool_exhaustion_rolls_back(small_ctx):
    a = small_ctx.stream_alloc(2000)
    b = small_ctx.stream_alloc(2000)
    free0 = small_ctx.free_pages()
    small_ctx.fill_synthetic(a, 16 * (free0 - 1), 1)
    assert small_ctx.free_pages() == 1
    x = np.zeros((2, 512), np.float32)
    with pytest.raises(rt.CudaError) as e:  # a needs a new page, b needs its first
        small_ctx.step([b, a], [0, 16 * (free0 - 1)], x)
    assert e.value.status == rt.POOL_EXHAUSTED
    assert small_ctx.free_pages() == 1 and small_ctx.length(b) == 0
    small_ctx.step([b], [0], x[:1])
    assert small_ctx.free_pages() == 0
    small_ctx.stream_free(a)
    small_ctx.stream_free(b)
    assert small_ctx.free_pages() == free0


def test_request_isolation(small_ctx):
    """tests/test_phonon_transformer.c:834-855 on the batched API: a stream's
    output depends only on its own history."""
    a, b, r = (small_ctx.stream_alloc(8) for _ in range(3))
    g = synth.Generator(9)
    x0, xb, x1 = g.normal(512), g.normal(512), g.normal(512)
    small_ctx.step([a, b], [0, 0], np.stack([x0, xb]))
    ya = small_ctx.step([a, b], [1, 1], np.stack([x1, x1]))[0]
    small_ctx.step([r], [0], x0[None])
    yr = small_ctx.step([r], [1], x1[None])[0]
    assert rt.rel_err(ya, yr) < 1e-5
    for s in (a, b, r):
        small_ctx.stream_free(s)

"""The benchmark's headline configuration against the CPU oracle, layer by layer.

512 streams in one decode step on the default batch paths, so the
step runs as two concurrent half batches (two lanes), with the projections on
the tcgen05 tensor cores (digit-sliced int8), bf16 K/V pages and contexts
U[64, 2048] (seed 2, the bench's own draw). A second case runs 192 streams on
one lane, where attention hands out its chunks by ticket (guided
self-scheduling). Three steps each; 32 (16) streams spread over both halves,
the longest and shortest contexts included, are teacher-forced through every
layer against the oracle's bf16-K/V mode (tests/parity.py) and bounded at
1e-4 per layer (max relative error with the 1e-2 floor); the normwise error
is reported beside it. The appended K/V rows must equal the oracle's up to
one bf16 rounding flip (the device sums its projections in another order)."""
import numpy as np
import pytest

from phonon_b200 import runtime as rt
from phonon_b200 import synth

import parity

pytestmark = pytest.mark.gpu
STEPS = 3


def _contexts(n, seed=2):
    """The bench's initial prefix draw (ServingSim): U[64, 2048], seed 2."""
    rng = np.random.default_rng(seed)
    return [int(rng.integers(64, 2048 + 1)) for _ in range(n)]


def _select(lens, n_pick):
    n = len(lens)
    half = n // 2
    picks = set()
    for lo, hi in ((0, half), (half, n)):
        idx = np.arange(lo, hi)
        picks.update(int(i) for i in idx[np.linspace(0, len(idx) - 1, n_pick // 2 - 1).astype(int)])
        seg = np.asarray(lens[lo:hi])
        picks.add(lo + int(np.argmax(seg)))
        picks.add(lo + int(np.argmin(seg)))
    return sorted(picks)


@pytest.mark.parametrize("n,n_pick", [(512, 32), (192, 16)])
def test_headline_step_teacher_forced(cuda_ok, oracle, weights12, n, n_pick):
    lens = _contexts(n)
    pages = sum((ln + STEPS) // 16 + 1 for ln in lens) + 64
    ctx = rt.Context(weights12, max_streams=n + 8, max_batch=n, pool_pages=pages, kv_type=rt.KV_BF16)
    if n < 512:  # one lane, so that attention hands out its chunks by ticket
        ctx.set_batch_paths(split_min_batch=1 << 20)
    trace = parity.Trace(ctx, n)
    try:
        streams = [ctx.stream_alloc(2048 + STEPS + 16) for _ in range(n)]
        for i, (s, ln) in enumerate(zip(streams, lens)):
            ctx.fill_synthetic(s, ln, 1000003 * i + 17)
        g = synth.Generator(2024 + n)
        xs, traces, positions = [], [], []
        for t in range(STEPS):
            pos = [ln + t for ln in lens]
            x = g.normal(n * 512).reshape(n, 512)
            y = ctx.step(streams, pos, x)
            tr = trace.read(n)
            assert np.array_equal(tr[-1], y)  # the last layer's rows are the step's output
            xs.append(x)
            traces.append(tr)
            positions.append(pos)
        om = oracle.model(weights12)
        stats = parity.Stats()
        picks = _select(lens, n_pick)
        assert any(i >= n // 2 for i in picks) and int(np.argmax(lens)) in picks
        for i in picks:
            parity.check_stream_oracle(ctx, om, streams[i], [p[i] for p in positions], [x[i] for x in xs],
                                       traces, i, stats, kv_bf16=True, label=f"stream {i} ctx {lens[i]}")
        print(f"{n} streams ({len(picks)} checked, contexts {min(lens)}..{max(lens)}): {stats}")
        assert stats.rel < parity.PER_LAYER_TOL, str(stats)
        assert stats.kv_rel < 1e-2 and stats.kv_flips <= max(8, stats.kv_elems // 1000), str(stats)
    finally:
        trace.close()
        ctx.close()

"""Serving failover on libphonon_cuda workers (one GPU, several contexts).

A worker whose step call raises (a host-side fault; nothing faults on the
GPU) is taken out of service, and its streams are re-prefilled from their
input history on the other contexts. The outputs of every stream, before
and after the move, agree with an undisturbed single-context run within the
final-output tolerance of the reference's tests (the re-prefill runs the
batched prefill path, and batches of other compositions merge attention
splits in another order)."""
import numpy as np
import pytest

from phonon_b200 import runtime as rt
from phonon_b200 import serving, synth

pytestmark = pytest.mark.gpu
FINAL_TOL = 1e-3


class FailingWorker(serving.CudaWorker):
    def __init__(self, ctx, capacity, fail_at):
        super().__init__(ctx, capacity)
        self.fail_at, self.calls = fail_at, 0

    def step(self, sids, x):
        self.calls += 1
        if self.calls >= self.fail_at:
            raise RuntimeError("injected worker failure")
        return super().step(sids, x)


def _inputs(sid, position):
    return synth.Generator(77 + 7919 * sid + position).normal(512).astype(np.float32)


def _run(server, prefixes, steps):
    outs = {}
    for sid, n in prefixes.items():
        server.open(sid, np.stack([_inputs(sid, p) for p in range(n)]))
    for k in range(steps):
        y = server.step({sid: _inputs(sid, n + k) for sid, n in prefixes.items()})
        for sid, n in prefixes.items():
            outs[(sid, n + k)] = y[sid]
    return outs


def test_cuda_failover(cuda_ok, weights12):
    prefixes = {0: 12, 1: 40, 2: 5, 3: 27, 4: 16, 5: 33}
    kw = dict(max_streams=16, max_batch=16, pool_pages=256, kv_type=rt.KV_F32)
    ctxs = [rt.Context(weights12, **kw) for _ in range(4)]
    try:
        ref = _run(serving.ShardedServer([serving.CudaWorker(ctxs[0], 128)]), prefixes, 8)
        bad = FailingWorker(ctxs[2], 128, fail_at=3)
        server = serving.ShardedServer([serving.CudaWorker(ctxs[1], 128), bad, serving.CudaWorker(ctxs[3], 128)])
        outs = _run(server, prefixes, 8)
        assert server.failed == [1] and server.migrations == len(bad.slot)
        worst = max(rt.rel_err(outs[k], y) for k, y in ref.items())
        assert worst < FINAL_TOL, worst
    finally:
        for c in ctxs:
            c.close()

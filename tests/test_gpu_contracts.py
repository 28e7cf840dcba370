"""Failure, cancel and argument contracts of the C ABI (no GPU fault is
provoked: non-finite values and cancellation are host-made)."""
import numpy as np
import pytest

from phonon_b200 import runtime as rt
from phonon_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx(cuda_ok):
    w = synth.flow_weights(3, seed=6)
    c = rt.Context(w, max_streams=8, max_batch=8, pool_pages=64)
    yield c
    c.close()


def test_nonfinite_input_fails_only_that_stream(ctx):
    a, b = ctx.stream_alloc(32), ctx.stream_alloc(32)
    x = synth.Generator(1).normal(1024).reshape(2, 512)
    x[1, 17] = np.nan
    y, status = ctx.step([a, b], [0, 0], x, raise_on_status=False)
    assert status[0] == rt.OK and status[1] == rt.NON_FINITE
    assert ctx.length(a) == 1 and ctx.length(b) == 0
    assert not y[1].any()  # output untouched on failure
    ctx.step([b], [0], x[:1])  # the failed position can be retried
    assert ctx.length(b) == 1
    ctx.stream_free(a)
    ctx.stream_free(b)


def test_pinned_host_buffers(ctx):
    """Page-locked x goes to the device by DMA without the staging copy, and
    an `out` buffer receives y: results equal those of plain numpy buffers,
    and a failed stream's row of `out` is left as it was."""
    import torch
    g = synth.Generator(11)
    x = g.normal(3 * 512).reshape(3, 512).astype(np.float32)
    x[2, 5] = np.inf
    pinned_x = torch.from_numpy(x).pin_memory().numpy()
    pinned_y = torch.full((3, 512), 7.0).pin_memory().numpy()
    a = [ctx.stream_alloc(32) for _ in range(3)]
    b = [ctx.stream_alloc(32) for _ in range(3)]
    for pos in range(3):
        y_ref, st_ref = ctx.step(b, [pos, pos, 0], x, raise_on_status=False)
        y, st = ctx.step(a, [pos, pos, 0], pinned_x, raise_on_status=False, out=pinned_y)
        assert y is pinned_y
        assert list(st) == list(st_ref) == [rt.OK, rt.OK, rt.NON_FINITE]
        assert np.array_equal(pinned_y[:2], y_ref[:2])
        assert np.all(pinned_y[2] == 7.0)
    for s in a + b:
        ctx.stream_free(s)


def test_argument_checks(ctx):
    a = ctx.stream_alloc(4)
    x = np.zeros((2, 512), np.float32)
    for streams, pos, code in (([a], [1], rt.BAD_POSITION), ([a, a], [0, 0], rt.INVALID),
                               ([a], [4], rt.CAPACITY), ([99], [0], rt.INVALID)):
        with pytest.raises(rt.CudaError) as e:
            ctx.step(streams, pos, x[:len(streams)])
        assert e.value.status == code
    assert ctx.length(a) == 0
    ctx.stream_free(a)


@pytest.mark.parametrize("stop", [1, 2, 3, 4])
def test_cancel_polls_and_resets(ctx, stop):
    a = ctx.stream_alloc(16)
    g = synth.Generator(2)
    ctx.step([a], [0], g.normal(512)[None])
    calls = []

    def poll(_):
        calls.append(1)
        return 1 if len(calls) == stop else 0

    with pytest.raises(rt.CudaError) as e:
        ctx.step([a], [1], g.normal(512)[None], cancel=poll)
    assert e.value.status == rt.CANCELLED and len(calls) == stop
    assert ctx.length(a) == 0 and len(ctx.pages(a)) == 0  # cache reset
    ctx.stream_free(a)


def test_cancel_never_fires_polls_layers_plus_one(ctx):
    a = ctx.stream_alloc(16)
    calls = []
    ctx.step([a], [0], np.ones((1, 512), np.float32), cancel=lambda _: calls.append(1) or 0)
    assert len(calls) == 3 + 1 and ctx.length(a) == 1
    ctx.stream_free(a)


def test_append_contracts(ctx):
    a = ctx.stream_alloc(8)
    rows = synth.Generator(3).normal(3 * 512).reshape(3, 512)
    with pytest.raises(rt.CudaError):
        ctx.append(a, np.zeros((9, 512), np.float32))  # longer than capacity
    bad = rows.copy()
    bad[2, 0] = np.inf
    with pytest.raises(rt.CudaError) as e:
        ctx.append(a, bad)
    assert e.value.status == rt.NON_FINITE and ctx.length(a) == 0
    ctx.append(a, rows)
    assert ctx.length(a) == 3
    with pytest.raises(rt.CudaError) as e:
        ctx.append(a, rows)  # cache must be empty
    assert e.value.status == rt.BAD_POSITION
    ctx.stream_free(a)

"""Bounded device waits expire cleanly (no GPU fault is made).

A wait on something nothing will ever complete (an mbarrier that no TMA
fills, a grid barrier one CTA never reaches) runs the library's own wait
routines with a short budget: the kernel must report the expiry through the
error flag, return, and leave the device usable for the next call."""
import numpy as np
import pytest

from phonon_b200 import runtime as rt

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", [0, 1, 2])
def test_wait_expires_and_reports(cuda_ok, kind):
    """kind 2: the expiry reaches the status words of an allocation-free
    linear call (phonon_cuda_linear_apply_device_noalloc) as DEVICE_ERROR."""
    st, secs = rt.wait_expiry_probe(kind, 2000)  # 2 ms budget
    assert st == rt.DEVICE_ERROR
    assert 0.001 < secs < 0.5, secs


def test_device_usable_after_expiry(cuda_ok, weights12):
    st, _ = rt.wait_expiry_probe(1, 1000)
    assert st == rt.DEVICE_ERROR
    ctx = rt.Context(weights12, max_streams=4, max_batch=4, pool_pages=64)
    try:
        s = ctx.stream_alloc(64)
        ctx.fill_synthetic(s, 20, 1)
        y = ctx.step([s], [20], np.ones((1, 512), np.float32))
        assert np.isfinite(y).all()
    finally:
        ctx.close()

"""phonon_cuda_linear_apply_device_noalloc: the allocation-free entry point.

Callers such as a real-time audio thread (where cudaMalloc may block past the
audio deadline) or an engine whose device memory was fixed at start-up cannot
call cudaMalloc mid-run. This entry point serves them: it keeps its scratch in
a device array that the library owns, and allocates nothing. Its output must
match the allocating entry point phonon_cuda_linear_apply_device on the same
inputs, within the per-layer tolerance of the parity tests, on two calls in a
row. The second call reuses the scratch the first one left behind. A row
with a non-finite value is flagged in its own status word only, and free
device memory is the same before and after a call."""
import ctypes as C

import numpy as np
import pytest

from phonon_b200 import runtime as rt
from phonon_b200 import synth

pytestmark = pytest.mark.gpu

NOALLOC_MAX_BATCH = 64


def noalloc_fn():
    L = rt.lib()
    fn = L.phonon_cuda_linear_apply_device_noalloc
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    fn.restype = C.c_int
    return fn


@pytest.mark.parametrize("rows,cols,batch", [(1536, 512, 64), (512, 2048, 40), (2048, 512, 7), (512, 512, 1)])
def test_noalloc_matches_allocating_entry_point(cuda_ok, rows, cols, batch):
    import torch
    g = synth.Generator(1000 + rows + cols)
    lin = rt.Linear(g.q8_linear(rows, cols, synth.SCALE_PER_ROW), rows, cols)
    bias = torch.tensor(g.normal(rows), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    fn = noalloc_fn()
    for call in range(2):  # two calls in a row share the scratch
        x = torch.tensor(g.normal(batch * cols).reshape(batch, cols), device="cuda")
        y_ref = torch.empty(batch, rows, device="cuda")
        y_new = torch.full((batch, rows), float("nan"), device="cuda")
        st_ref = torch.zeros(batch, dtype=torch.int32, device="cuda")
        st_new = torch.zeros(batch, dtype=torch.int32, device="cuda")
        lin.apply_device(x.data_ptr(), batch, y_ref.data_ptr(), stream, bias.data_ptr(), st_ref.data_ptr())
        rc = fn(lin.h, x.data_ptr(), batch, bias.data_ptr(), y_new.data_ptr(), st_new.data_ptr(), stream)
        assert rc == rt.OK, rt.lib().phonon_cuda_status_string(rc)
        torch.cuda.synchronize()
        a, b = y_new.cpu().numpy().ravel(), y_ref.cpu().numpy().ravel()
        assert not st_new.any() and not st_ref.any()
        assert rt.rel_err(a, b) < 1e-4, (call, rt.rel_err(a, b))
        assert np.abs(a - b).max() / np.abs(b).max() < 1e-5
    lin.close()


def test_noalloc_limits(cuda_ok):
    import torch
    g = synth.Generator(7)
    fn = noalloc_fn()
    lin = rt.Linear(g.q8_linear(512, 512, synth.SCALE_PER_ROW), 512, 512)
    x = torch.zeros(NOALLOC_MAX_BATCH + 1, 512, device="cuda")
    y = torch.zeros(NOALLOC_MAX_BATCH + 1, 512, device="cuda")
    rc = fn(lin.h, x.data_ptr(), NOALLOC_MAX_BATCH + 1, None, y.data_ptr(), None, None)
    assert rc == rt.CAPACITY
    bf = rt.Linear(np.zeros(512 * 512, np.uint16), 512, 512, kind=rt.BF16)
    rc = fn(bf.h, x.data_ptr(), 4, None, y.data_ptr(), None, None)
    assert rc == rt.INVALID  # only Q8_0 with one scale per row runs on this path
    lin.close()
    bf.close()


def test_noalloc_nonfinite_row_and_no_allocation(cuda_ok):
    """Row 3 of 9 holds a NaN: only its status word is flagged (the other
    rows match the allocating entry point), and a call leaves the device's
    free memory unchanged."""
    import torch
    g = synth.Generator(99)
    rows, cols, batch, bad = 512, 2048, 9, 3
    lin = rt.Linear(g.q8_linear(rows, cols, synth.SCALE_PER_ROW), rows, cols)
    stream = torch.cuda.current_stream().cuda_stream
    fn = noalloc_fn()
    x = torch.tensor(g.normal(batch * cols).reshape(batch, cols), device="cuda")
    x[bad, 17] = float("nan")
    y_ref = torch.empty(batch, rows, device="cuda")
    y_new = torch.empty(batch, rows, device="cuda")
    st_ref = torch.zeros(batch, dtype=torch.int32, device="cuda")
    st_new = torch.zeros(batch, dtype=torch.int32, device="cuda")
    lin.apply_device(x.data_ptr(), batch, y_ref.data_ptr(), stream, None, st_ref.data_ptr())
    assert fn(lin.h, x.data_ptr(), batch, None, y_new.data_ptr(), st_new.data_ptr(), stream) == rt.OK
    torch.cuda.synchronize()
    flagged = st_new.cpu().numpy()
    assert flagged[bad] == rt.NON_FINITE and np.count_nonzero(flagged) == 1, flagged
    assert st_ref.cpu().numpy()[bad] == rt.NON_FINITE
    ok = [i for i in range(batch) if i != bad]
    a, b = y_new.cpu().numpy()[ok], y_ref.cpu().numpy()[ok]
    assert rt.rel_err(a.ravel(), b.ravel()) < 1e-4
    st_new.zero_()
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    assert fn(lin.h, x.data_ptr(), batch, None, y_new.data_ptr(), st_new.data_ptr(), stream) == rt.OK
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    lin.close()

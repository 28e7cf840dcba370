"""The C17 drop-in (libphonon_transformer_cuda.so) under the reference API:
the model-free contracts of speech-mac tests/test_phonon_transformer.c:586-855,
tests/test_phonon_q8.c and tests/test_speech.c:279-306, restated in Python."""
import ctypes as C

import numpy as np
import pytest

from phonon_b200._libs import load_dropin

pytestmark = pytest.mark.gpu


class View(C.Structure):  # PhononTensorView
    _fields_ = [("dtype", C.c_int), ("rank", C.c_uint), ("shape", C.c_uint64 * 8),
                ("data", C.c_void_p), ("byte_count", C.c_size_t), ("linear_data", C.c_void_p)]


class LayerWeights(C.Structure):  # PhononFlowLayerWeights
    _fields_ = [(n, C.POINTER(View)) for n in ("qkv", "attention_out", "mlp_in", "mlp_out",
                                               "norm1_weight", "norm1_bias", "norm2_weight",
                                               "norm2_bias")]


class KvCache(C.Structure):  # PhononKvCache
    _fields_ = [("capacity", C.c_size_t), ("length", C.c_size_t),
                ("keys", C.POINTER(C.c_float)), ("values", C.POINTER(C.c_float))]


POLL = C.CFUNCTYPE(C.c_int, C.c_void_p)


def p(a):
    return a.ctypes.data_as(C.c_void_p)


@pytest.fixture(scope="module")
def lib(cuda_ok):
    L = load_dropin()
    V, K = C.POINTER(View), C.POINTER(KvCache)
    L.phonon_kv_cache_init.argtypes = [K, C.c_size_t]
    L.phonon_kv_cache_reset.argtypes = [K]
    L.phonon_kv_cache_destroy.argtypes = [K]
    L.phonon_kv_cache_append.argtypes = [K, C.c_size_t, C.c_size_t, C.c_void_p, C.c_void_p, C.c_size_t]
    L.phonon_kv_cache_commit_position.argtypes = [K, C.c_size_t]
    L.phonon_linear.argtypes = [V, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_void_p]
    L.phonon_q8_dot.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]
    L.phonon_q8_matvec.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p]
    W = C.POINTER(LayerWeights)
    L.phonon_flow_layer_step.argtypes = [W, K, C.c_size_t, C.c_size_t, C.c_void_p, C.c_float, C.c_void_p]
    L.phonon_flow_stack_step.argtypes = [W, K, C.c_size_t, C.c_void_p, C.c_float, C.c_void_p]
    L.phonon_flow_stack_step_cancel.argtypes = [W, K, C.c_size_t, C.c_void_p, C.c_float, C.c_void_p,
                                                POLL, C.c_void_p]
    L.phonon_flow_stack_prefill.argtypes = [W, K, C.c_void_p, C.c_size_t, C.c_float, C.c_void_p]
    L.phonon_flow_stack_prefill_cancel.argtypes = [W, K, C.c_void_p, C.c_size_t, C.c_float,
                                                   C.c_void_p, POLL, C.c_void_p]
    L.phonon_erf_gelu.argtypes = [C.c_void_p, C.c_size_t]
    return L


def view(dtype, shape, data):
    v = View()
    v.dtype, v.rank = dtype, len(shape)
    for i, s in enumerate(shape):
        v.shape[i] = s
    v.data = data.ctypes.data
    v.byte_count = data.nbytes
    return v


def new_cache(lib, capacity):
    c = KvCache()
    assert lib.phonon_kv_cache_init(C.byref(c), capacity)
    return c


def test_kv_layout_and_commit(lib):
    cache, other = new_cache(lib, 2), new_cache(lib, 2)
    k = np.arange(512, dtype=np.float32)
    v = -k
    assert lib.phonon_kv_cache_append(C.byref(cache), 8, 1, p(k), p(v), 512)
    assert cache.keys[(8 * 2 + 1) * 512 + 7] == 7.0 and cache.length == 0
    assert lib.phonon_kv_cache_commit_position(C.byref(cache), 0) and cache.length == 1
    assert not lib.phonon_kv_cache_commit_position(C.byref(cache), 0)
    assert other.length == 0
    assert not lib.phonon_kv_cache_append(C.byref(cache), 9, 0, p(k), p(v), 512)
    lib.phonon_kv_cache_reset(C.byref(cache))
    assert cache.length == 0
    lib.phonon_kv_cache_destroy(C.byref(cache))
    lib.phonon_kv_cache_destroy(C.byref(other))
    assert not cache.keys and not cache.values


def _block(scale, values):
    b = np.zeros(34, np.uint8)
    b[0], b[1] = scale & 0xFF, scale >> 8
    b[2:] = np.asarray(values, np.int8).view(np.uint8)
    return b


def test_q8_api(lib):
    blocks = np.concatenate([_block(0x3800, np.arange(32) - 16), _block(0x4000, np.ones(32))])
    ones = np.ones(64, np.float32)
    out = C.c_float()
    assert lib.phonon_q8_dot(p(blocks), p(ones), 64, C.byref(out)) and out.value == 56.0
    assert not lib.phonon_q8_dot(p(blocks), p(ones), 63, C.byref(out))
    y = np.zeros(2, np.float32)
    m = np.concatenate([blocks, blocks[34:], blocks[:34]])
    assert lib.phonon_q8_matvec(p(m), p(ones), 2, 64, p(y)) and list(y) == [56.0, 56.0]
    assert not lib.phonon_q8_matvec(p(m), p(ones), 2, 64, p(ones))  # output overlaps input
    bad = blocks.copy()
    bad[0], bad[1] = 0x00, 0x7C
    assert not lib.phonon_q8_dot(p(bad), p(ones), 32, C.byref(out))


def test_linear_api(lib):
    w = np.array([0x3F80, 0xC000, 0x4000, 0x3F00], np.uint16)
    v = view(2, (2, 2), w)
    y = np.zeros(2, np.float32)
    assert lib.phonon_linear(C.byref(v), p(np.array([3.0, 2.0], np.float32)), 2, 2, None, p(y))
    assert list(y) == [-1.0, 7.0]
    ones = np.full(64, 0x3F80, np.uint16)
    x = np.ones(32, np.float32)
    bias = np.array([np.nan, 0.25], np.float32)
    vc = view(2, (2, 32), ones)
    assert not lib.phonon_linear(C.byref(vc), p(x), 2, 32, p(bias), p(y))
    ones[0] = 0x7F80
    assert not lib.phonon_linear(C.byref(vc), p(x), 2, 32, None, p(y))
    ones[0] = 0x3F80
    vc.byte_count -= 1
    assert not lib.phonon_linear(C.byref(vc), p(x), 2, 32, None, p(y))
    q8 = np.concatenate([_block(0x0001, np.ones(32)), _block(0x8000, np.ones(32))])
    vq = view(1, (2, 32), q8)
    assert lib.phonon_linear(C.byref(vq), p(x), 2, 32, None, p(y))
    assert list(y) == [2.0 ** -19, 0.0]
    q8[0], q8[1] = 0x00, 0x7E
    assert not lib.phonon_linear(C.byref(vq), p(x), 2, 32, None, p(y))


class ZeroStack:
    """BF16 zero projections and unit norms: every layer is the identity
    (tests/test_phonon_transformer.c:707-747)."""

    def __init__(self):
        self.mats = [np.zeros(n, np.uint16) for n in (1536 * 512, 512 * 512, 2048 * 512, 512 * 2048)]
        shapes = ((1536, 512), (512, 512), (2048, 512), (512, 2048))
        self.views = [view(2, s, m) for s, m in zip(shapes, self.mats)]
        self.ones = np.full(512, 0x3F80, np.uint16)
        self.zeros = np.zeros(512, np.uint16)
        self.nw, self.nb = view(2, (512,), self.ones), view(2, (512,), self.zeros)
        self.layer = LayerWeights(*[C.pointer(v) for v in self.views],
                                  C.pointer(self.nw), C.pointer(self.nb),
                                  C.pointer(self.nw), C.pointer(self.nb))
        self.stack = (LayerWeights * 9)(*[self.layer] * 9)


@pytest.fixture(scope="module")
def zs():
    return ZeroStack()


def test_identity_layer_and_stack(lib, zs):
    state = (np.arange(512, dtype=np.float32) / 512.0)
    nxt = np.zeros(512, np.float32)
    cache = new_cache(lib, 2)
    assert lib.phonon_flow_layer_step(C.byref(zs.layer), C.byref(cache), 0, 0, p(state), 10000.0, p(nxt))
    assert np.array_equal(nxt, state)
    assert lib.phonon_flow_stack_step(zs.stack, C.byref(cache), 0, p(state), 10000.0, p(nxt))
    assert cache.length == 1 and np.array_equal(nxt, state)
    assert lib.phonon_flow_stack_step(zs.stack, C.byref(cache), 1, p(state), 10000.0, p(nxt))
    assert cache.length == 2
    lib.phonon_kv_cache_destroy(C.byref(cache))


def test_prefill_contracts(lib, zs):
    state = (np.arange(512, dtype=np.float32) / 512.0)
    rows = np.concatenate([state, -np.arange(512, dtype=np.float32) / 256.0])
    out = np.zeros(512, np.float32)
    a, b = new_cache(lib, 2), new_cache(lib, 2)
    for bad_len in (0, 3, 8193):
        assert not lib.phonon_flow_stack_prefill(zs.stack, C.byref(a), p(rows), bad_len, 10000.0, p(out))
    assert lib.phonon_flow_stack_prefill(zs.stack, C.byref(a), p(rows), 2, 10000.0, p(out))
    assert a.length == 2 and b.length == 0 and np.array_equal(out, rows[512:])
    assert not lib.phonon_flow_stack_prefill(zs.stack, C.byref(a), p(rows), 1, 10000.0, p(out))
    assert a.length == 2
    lib.phonon_kv_cache_reset(C.byref(a))
    out[0] = 123.0
    rows[0] = np.nan
    assert not lib.phonon_flow_stack_prefill(zs.stack, C.byref(a), p(rows), 2, 10000.0, p(out))
    assert a.length == 0 and out[0] == 123.0
    rows[0] = 0.0
    assert lib.phonon_flow_stack_prefill(zs.stack, C.byref(a), p(rows), 1, 10000.0, p(out))
    assert a.length == 1
    assert lib.phonon_flow_stack_step(zs.stack, C.byref(a), 1, p(state), 10000.0, p(out))
    assert a.length == 2 and b.length == 0
    lib.phonon_kv_cache_destroy(C.byref(a))
    lib.phonon_kv_cache_destroy(C.byref(b))


def test_cancel_counts(lib, zs):
    """tests/test_speech.c:293-306: the stop-th poll cancels, the cache is
    reset and the output stays untouched."""
    out = np.full(512, 123.0, np.float32)
    cond = np.zeros(512, np.float32)
    cache = new_cache(lib, 2)
    calls = []

    def make(stop):
        calls.clear()
        return POLL(lambda _: (calls.append(1), 1 if len(calls) == stop else 0)[1])

    poll = make(3)
    assert not lib.phonon_flow_stack_step_cancel(zs.stack, C.byref(cache), 0, p(cond), 10000.0,
                                                 p(out), poll, None)
    assert len(calls) == 3 and cache.length == 0 and np.all(out == 123.0)
    poll = make(4)
    assert not lib.phonon_flow_stack_prefill_cancel(zs.stack, C.byref(cache), p(cond), 1, 10000.0,
                                                    p(out), poll, None)
    assert len(calls) == 4 and cache.length == 0 and np.all(out == 123.0)
    poll = make(10 ** 6)
    assert lib.phonon_flow_stack_step_cancel(zs.stack, C.byref(cache), 0, p(cond), 10000.0, p(out),
                                             poll, None)
    assert len(calls) == 10 and cache.length == 1  # 9 layers + 1, like the reference
    lib.phonon_kv_cache_destroy(C.byref(cache))


def test_causal_dependence_and_isolation(lib):
    """Nonzero V[0,0] and out[0,0] make attention observably causal; requests
    stay isolated (tests/test_phonon_transformer.c:822-855)."""
    z = ZeroStack()
    z.mats[0][1024 * 512] = 0x3F80
    z.mats[1][0] = 0x3F80
    first = np.zeros(512, np.float32)
    second = np.zeros(512, np.float32)
    first[0], second[0] = 1.0, 3.0
    o0, o1 = np.zeros(512, np.float32), np.zeros(512, np.float32)
    causal = new_cache(lib, 2)
    assert lib.phonon_flow_stack_step(z.stack, C.byref(causal), 0, p(first), 10000.0, p(o0))
    assert lib.phonon_flow_stack_step(z.stack, C.byref(causal), 1, p(second), 10000.0, p(o1))
    assert o0[0] > 1.0 and o1[0] > 3.0
    lib.phonon_kv_cache_destroy(C.byref(causal))
    ra, rb, rr = (new_cache(lib, 2) for _ in range(3))
    div, shared = np.zeros(512, np.float32), np.zeros(512, np.float32)
    div[0], shared[0] = 1.0, 3.0
    aout, bout, rout = (np.zeros(512, np.float32) for _ in range(3))
    assert lib.phonon_flow_stack_step(z.stack, C.byref(ra), 0, p(div), 10000.0, p(aout))
    div[0] = -7.0
    assert lib.phonon_flow_stack_step(z.stack, C.byref(rb), 0, p(div), 10000.0, p(bout))
    assert lib.phonon_flow_stack_step(z.stack, C.byref(ra), 1, p(shared), 10000.0, p(aout))
    one = np.zeros(512, np.float32)
    one[0] = 1.0
    assert lib.phonon_flow_stack_step(z.stack, C.byref(rr), 0, p(one), 10000.0, p(rout))
    assert lib.phonon_flow_stack_step(z.stack, C.byref(rr), 1, p(shared), 10000.0, p(rout))
    assert np.abs(aout - rout).max() < 1e-6
    lib.phonon_kv_cache_reset(C.byref(ra))
    assert lib.phonon_flow_stack_step(z.stack, C.byref(ra), 0, p(one), 10000.0, p(aout))
    assert ra.length == 1 and abs(aout[0] - bout[0]) > 1e-4
    for c in (ra, rb, rr):
        lib.phonon_kv_cache_destroy(C.byref(c))


def test_mirror_tracks_device_rows(lib, zs):
    """After a device step the host keys/values mirror holds the appended rows
    (zero projections: K = V = 0 after RoPE of 0)."""
    cache = new_cache(lib, 4)
    k = np.full(512, 5.0, np.float32)
    assert lib.phonon_kv_cache_append(C.byref(cache), 0, 0, p(k), p(k), 512)
    x, out = np.ones(512, np.float32), np.zeros(512, np.float32)
    assert lib.phonon_flow_stack_step(zs.stack, C.byref(cache), 0, p(x), 10000.0, p(out))
    assert cache.keys[0] == 0.0  # the step overwrote position 0 with its own K
    lib.phonon_kv_cache_destroy(C.byref(cache))

"""ctypes bindings of libphonon_cuda (include/phonon_cuda.h).

Thin Python mirror of the C ABI for tests and the benchmark. The library is
loaded from the package directory; a missing library raises instead of
falling back to anything else.
"""
import ctypes as C

import numpy as np

from ._libs import load_cuda

KERNEL_CLASSES = ("qkv", "attention", "combine", "out", "up", "down", "other", "fused", "head")
OK, INVALID, NON_FINITE, OOM, POOL_EXHAUSTED, CAPACITY, BAD_POSITION, CANCELLED, DEVICE_ERROR = range(9)
Q8_0, BF16 = 1, 2
KV_F32, KV_BF16 = 0, 1
FUSED_MAX_BATCH = 64  # PHONON_CUDA_FUSED_MAX_BATCH
MAX_POSITIONS = 8192  # PHONON_CUDA_MAX_POSITIONS
WIDTH = 512
PAGE = 16

CANCEL_FN = C.CFUNCTYPE(C.c_int, C.c_void_p)


class Config(C.Structure):
    _fields_ = [("device", C.c_int), ("n_layers", C.c_uint32), ("max_streams", C.c_uint32),
                ("max_batch", C.c_uint32), ("pool_pages", C.c_uint32), ("kv_type", C.c_uint32),
                ("theta", C.c_float)]


class Layer(C.Structure):
    _fields_ = [("qkv", C.c_void_p), ("attention_out", C.c_void_p), ("mlp_in", C.c_void_p),
                ("mlp_out", C.c_void_p), ("norm1_weight", C.c_void_p), ("norm1_bias", C.c_void_p),
                ("norm2_weight", C.c_void_p), ("norm2_bias", C.c_void_p),
                ("linear_kind", C.c_uint32)]


HEAD_BLOCKS = 6  # PHONON_CUDA_HEAD_BLOCKS
LATENT = 32  # PHONON_CUDA_LATENT


class Affine(C.Structure):
    _fields_ = [("weight", C.c_void_p), ("bias", C.c_void_p)]


class HeadWeights(C.Structure):
    _fields_ = [("input", Affine), ("cond", Affine), ("time", (Affine * 2) * 2),
                ("time_freqs", C.c_void_p * 2), ("time_alpha", C.c_void_p * 2),
                ("block_ada", Affine * HEAD_BLOCKS), ("block_norm_w", C.c_void_p * HEAD_BLOCKS),
                ("block_norm_b", C.c_void_p * HEAD_BLOCKS), ("block_mlp", (Affine * 2) * HEAD_BLOCKS),
                ("final_ada", Affine), ("final_out", Affine), ("eos", Affine), ("embed", C.c_void_p),
                ("out_norm_w", C.c_void_p), ("out_norm_b", C.c_void_p)]


class MimiWeights(C.Structure):
    _fields_ = [("projection", C.c_void_p), ("upsample", C.c_void_p), ("in_proj", C.c_void_p * 2),
                ("out_proj", C.c_void_p * 2), ("linear1", C.c_void_p * 2), ("linear2", C.c_void_p * 2),
                ("norm1_w", C.c_void_p * 2), ("norm1_b", C.c_void_p * 2), ("norm2_w", C.c_void_p * 2),
                ("norm2_b", C.c_void_p * 2), ("scale1", C.c_void_p * 2), ("scale2", C.c_void_p * 2)]


class CudaError(RuntimeError):
    def __init__(self, status, what):
        self.status = status
        super().__init__(f"{what}: {lib().phonon_cuda_status_string(status).decode()} ({status})")


_typed = None


def lib():
    global _typed
    L = load_cuda()
    if _typed is L:
        return L
    P, U32, I32, SZ, F = C.c_void_p, C.c_uint32, C.c_int32, C.c_size_t, C.c_float
    sig = {
        "phonon_cuda_create": [C.POINTER(Config), C.POINTER(Layer), C.POINTER(P)],
        "phonon_cuda_set_layer": [P, U32, C.POINTER(Layer)],
        "phonon_cuda_set_theta": [P, F],
        "phonon_cuda_stream_alloc": [P, U32, C.POINTER(U32)],
        "phonon_cuda_stream_reset": [P, U32],
        "phonon_cuda_stream_free": [P, U32],
        "phonon_cuda_stream_length": [P, U32, C.POINTER(U32)],
        "phonon_cuda_stream_pages": [P, U32, P, U32, C.POINTER(U32)],
        "phonon_cuda_step": [P, U32, P, P, P, P, P, CANCEL_FN, P],
        "phonon_cuda_step_device": [P, U32, P, P, P, P],
        "phonon_cuda_sync": [P, P],
        "phonon_cuda_layer_step": [P, U32, U32, U32, P, P],
        "phonon_cuda_commit": [P, U32, U32],
        "phonon_cuda_append": [P, U32, P, U32, P, CANCEL_FN, P],
        "phonon_cuda_kv_read": [P, U32, U32, U32, U32, U32, P, P],
        "phonon_cuda_kv_write": [P, U32, U32, U32, U32, U32, P, P],
        "phonon_cuda_stream_fill_synthetic": [P, U32, U32, C.c_uint64],
        "phonon_cuda_linear_create": [C.c_int, C.c_int, P, SZ, SZ, C.POINTER(P)],
        "phonon_cuda_linear_apply": [P, P, SZ, P, P],
        "phonon_cuda_linear_apply_device": [P, P, SZ, P, P, P, P],
        "phonon_cuda_layer_norm": [C.c_int, P, P, P, SZ, F, P],
        "phonon_cuda_rms_norm": [C.c_int, P, P, SZ, F, P],
        "phonon_cuda_erf_gelu": [C.c_int, P, SZ],
        "phonon_cuda_rope_interleaved": [C.c_int, P, SZ, SZ, SZ, F],
        "phonon_cuda_profile_enable": [P, C.c_int],
        "phonon_cuda_profile_read": [P, P, P, P],
        "phonon_cuda_set_batch_paths": [P, U32, U32, U32, U32],
        "phonon_cuda_set_cluster_step": [P, U32, C.POINTER(C.c_int)],
        "phonon_cuda_set_layer_trace": [P, P, U32],
        "phonon_cuda_wait_expiry_probe": [C.c_int, C.c_int, U32, C.POINTER(C.c_uint64)],
        "phonon_cuda_head_create": [P, C.POINTER(HeadWeights), C.POINTER(P)],
        "phonon_cuda_head_forward": [P, U32, P, P, F, F, P],
        "phonon_cuda_head_set_tensor_min": [P, U32, C.POINTER(C.c_int)],
        "phonon_cuda_lsd_one_step": [P, U32, P, P, F, P],
        "phonon_cuda_eos_logit": [P, U32, P, P],
        "phonon_cuda_output_norm_device": [P, U32, P, P],
        "phonon_cuda_frame_step": [P, U32, P, P, P, P, P, F, P, P, P],
        "phonon_cuda_mimi_create": [C.c_int, C.POINTER(MimiWeights), U32, U32, C.POINTER(P)],
        "phonon_cuda_mimi_state_alloc": [P, C.POINTER(U32)],
        "phonon_cuda_mimi_state_reset": [P, U32],
        "phonon_cuda_mimi_state_free": [P, U32],
        "phonon_cuda_mimi_positions": [P, U32, C.POINTER(C.c_uint64)],
        "phonon_cuda_mimi_step": [P, U32, P, P, P, P],
        "phonon_cuda_mimi_set_tensor_min": [P, U32, C.POINTER(C.c_int)],
        "phonon_cuda_mimi_process": [P, U32, P, SZ, P, SZ],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = C.c_int
    L.phonon_cuda_mimi_destroy.argtypes = [P]
    L.phonon_cuda_mimi_destroy.restype = None
    L.phonon_cuda_head_free.argtypes = [P]
    L.phonon_cuda_head_free.restype = None
    L.phonon_cuda_destroy.argtypes = [P]
    L.phonon_cuda_destroy.restype = None
    L.phonon_cuda_linear_destroy.argtypes = [P]
    L.phonon_cuda_linear_destroy.restype = None
    L.phonon_cuda_linear_bytes.argtypes = [P]
    L.phonon_cuda_linear_bytes.restype = SZ
    L.phonon_cuda_free_pages.argtypes = [P]
    L.phonon_cuda_free_pages.restype = U32
    L.phonon_cuda_cuda_stream.argtypes = [P]
    L.phonon_cuda_cuda_stream.restype = P
    L.phonon_cuda_launch_count.argtypes = [P]
    L.phonon_cuda_launch_count.restype = C.c_uint64
    L.phonon_cuda_status_string.argtypes = [C.c_int]
    L.phonon_cuda_status_string.restype = C.c_char_p
    _typed = L
    return L


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def check(status, what):
    if status != OK:
        raise CudaError(status, what)


def wait_expiry_probe(kind, budget_us, device=0):
    """Run a bounded device wait on something nothing completes (kind 0: an
    mbarrier, 1: a grid barrier); returns (status, elapsed seconds)."""
    ns = C.c_uint64(0)
    st = lib().phonon_cuda_wait_expiry_probe(device, kind, budget_us, C.byref(ns))
    return st, ns.value * 1e-9


def rel_err(a, ref, floor=1e-2):
    """max_i |a_i - ref_i| / max(|ref_i|, floor * max_j |ref_j|)."""
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.maximum(np.abs(ref), floor * np.abs(ref).max())
    return float(np.max(np.abs(a - ref) / den))


def layer_struct(w, kind=Q8_0):
    return Layer(w["qkv"].ctypes.data, w["out"].ctypes.data, w["up"].ctypes.data,
                 w["down"].ctypes.data, w["norm1_w"].ctypes.data, w["norm1_b"].ctypes.data,
                 w["norm2_w"].ctypes.data, w["norm2_b"].ctypes.data, kind)


class Context:
    """One libphonon_cuda context (weights + KV page pool) on one device."""

    def __init__(self, weights, device=0, max_streams=64, max_batch=64, pool_pages=1024,
                 kv_type=KV_F32, theta=10000.0, kind=Q8_0):
        self.L = lib()
        self.n_layers = len(weights)
        layers = (Layer * self.n_layers)(*[layer_struct(w, kind) for w in weights])
        cfg = Config(device, self.n_layers, max_streams, max_batch, pool_pages, kv_type, theta)
        h = C.c_void_p()
        check(self.L.phonon_cuda_create(C.byref(cfg), layers, C.byref(h)), "phonon_cuda_create")
        self.h = h
        self.device = device
        self.kv_type = kv_type

    def close(self):
        if self.h:
            self.L.phonon_cuda_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # streams ----------------------------------------------------------------
    def stream_alloc(self, capacity):
        s = C.c_uint32()
        check(self.L.phonon_cuda_stream_alloc(self.h, capacity, C.byref(s)), "stream_alloc")
        return s.value

    def stream_free(self, s):
        check(self.L.phonon_cuda_stream_free(self.h, s), "stream_free")

    def stream_reset(self, s):
        check(self.L.phonon_cuda_stream_reset(self.h, s), "stream_reset")

    def length(self, s):
        n = C.c_uint32()
        check(self.L.phonon_cuda_stream_length(self.h, s, C.byref(n)), "stream_length")
        return n.value

    def pages(self, s):
        n = C.c_uint32()
        check(self.L.phonon_cuda_stream_pages(self.h, s, None, 0, C.byref(n)), "stream_pages")
        out = np.zeros(max(n.value, 1), np.int32)
        check(self.L.phonon_cuda_stream_pages(self.h, s, _p(out), n.value, C.byref(n)), "stream_pages")
        return out[:n.value]

    def free_pages(self):
        return self.L.phonon_cuda_free_pages(self.h)

    def fill_synthetic(self, s, length, seed):
        check(self.L.phonon_cuda_stream_fill_synthetic(self.h, s, length, seed), "fill_synthetic")

    # compute ----------------------------------------------------------------
    def step(self, streams, positions, x, cancel=None, raise_on_status=True, out=None):
        """One decode step through host buffers (phonon_cuda_step). `out`, if
        given, is a float32 C-contiguous [n][512] array that receives y (rows
        of failed streams are left as they were); x or out in page-locked
        memory (e.g. torch pin_memory tensors' numpy views) are copied by DMA
        directly."""
        n = len(streams)
        st = np.ascontiguousarray(streams, np.uint32)
        pos = np.ascontiguousarray(positions, np.uint32)
        x = np.ascontiguousarray(x, np.float32).reshape(n, WIDTH)
        if out is None:
            y = np.zeros((n, WIDTH), np.float32)
        else:
            y = out
            if y.dtype != np.float32 or y.shape != (n, WIDTH) or not y.flags.c_contiguous:
                raise ValueError("out must be a C-contiguous float32 array of shape (n, 512)")
        status = np.zeros(n, np.int32)
        cb = CANCEL_FN(cancel) if cancel else CANCEL_FN()
        rc = self.L.phonon_cuda_step(self.h, n, _p(st), _p(pos), _p(x), _p(y), _p(status), cb, None)
        check(rc, "phonon_cuda_step")
        if raise_on_status and status.any():
            raise CudaError(int(status[status != 0][0]), "phonon_cuda_step stream status")
        return y if raise_on_status else (y, status)

    def step_device(self, streams, positions, x_ptr, y_ptr):
        n = len(streams)
        st = np.ascontiguousarray(streams, np.uint32)
        pos = np.ascontiguousarray(positions, np.uint32)
        check(self.L.phonon_cuda_step_device(self.h, n, _p(st), _p(pos), C.c_void_p(x_ptr),
                                             C.c_void_p(y_ptr)), "phonon_cuda_step_device")

    def sync(self, n):
        status = np.zeros(n, np.int32)
        check(self.L.phonon_cuda_sync(self.h, _p(status)), "phonon_cuda_sync")
        return status

    def cuda_stream(self):
        return self.L.phonon_cuda_cuda_stream(self.h)

    def profile(self, enable=True):
        check(self.L.phonon_cuda_profile_enable(self.h, 1 if enable else 0), "profile_enable")

    def profile_read(self):
        n = len(KERNEL_CLASSES)
        ms, by = np.zeros(n, np.float64), np.zeros(n, np.float64)
        la = np.zeros(n, np.uint64)
        check(self.L.phonon_cuda_profile_read(self.h, _p(ms), _p(by), _p(la)), "profile_read")
        return {k: {"ms": float(ms[i]), "bytes": float(by[i]), "launches": int(la[i])}
                for i, k in enumerate(KERNEL_CLASSES)}

    def launch_count(self):
        return int(self.L.phonon_cuda_launch_count(self.h))

    def set_batch_paths(self, fused_min_batch=2, fused_max_batch=3, tensor_min_batch=4,
                        split_min_batch=96):
        """Batch sizes routed to the persistent whole-step launch
        (fused_min_batch..fused_max_batch; a minimum above the maximum
        disables it), to the tensor-core projections (>= tensor_min_batch) and
        to two concurrent half batches (>= split_min_batch)."""
        check(self.L.phonon_cuda_set_batch_paths(self.h, fused_min_batch, fused_max_batch, tensor_min_batch,
                                                 split_min_batch), "set_batch_paths")

    def set_cluster_step(self, max_position=8192):
        """Single-stream steps at positions below max_position run on one
        16-CTA cluster (0 disables it). Returns 0 when the context cannot run
        that path, 1 when it runs it with every projection on the CUDA cores,
        2 when its projections run on the tensor cores (weights with one
        scale per row)."""
        available = C.c_int(0)
        check(self.L.phonon_cuda_set_cluster_step(self.h, max_position, C.byref(available)), "set_cluster_step")
        return available.value

    def set_layer_trace(self, trace_ptr, max_rows):
        """Every later decode step also writes each layer's output rows into
        device memory at trace_ptr ([n_layers][max_rows][512] fp32); a null
        pointer (0 / None) switches the trace off."""
        check(self.L.phonon_cuda_set_layer_trace(self.h, C.c_void_p(trace_ptr or None),
                                                 max_rows if trace_ptr else 0), "set_layer_trace")

    def layer_step(self, s, layer, position, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros(WIDTH, np.float32)
        check(self.L.phonon_cuda_layer_step(self.h, s, layer, position, _p(x), _p(y)), "layer_step")
        return y

    def commit(self, s, position):
        check(self.L.phonon_cuda_commit(self.h, s, position), "commit")

    def append(self, s, rows, cancel=None):
        rows = np.ascontiguousarray(rows, np.float32)
        out = np.zeros(WIDTH, np.float32)
        cb = CANCEL_FN(cancel) if cancel else CANCEL_FN()
        check(self.L.phonon_cuda_append(self.h, s, _p(rows), rows.shape[0], _p(out), cb, None), "append")
        return out

    def kv_read(self, s, position, count=1, layer_begin=0, layer_count=None):
        lc = self.n_layers - layer_begin if layer_count is None else layer_count
        k = np.zeros((lc, count, WIDTH), np.float32)
        v = np.zeros((lc, count, WIDTH), np.float32)
        check(self.L.phonon_cuda_kv_read(self.h, s, layer_begin, lc, position, count, _p(k), _p(v)),
              "kv_read")
        return k, v

    def kv_write(self, s, position, keys, values, layer_begin=0):
        keys = np.ascontiguousarray(keys, np.float32)
        values = np.ascontiguousarray(values, np.float32)
        lc, count = keys.shape[0], keys.shape[1]
        check(self.L.phonon_cuda_kv_write(self.h, s, layer_begin, lc, position, count, _p(keys),
                                          _p(values)), "kv_write")


class Linear:
    """A device copy of one Q8_0 / bf16 matrix (phonon_cuda_linear_*)."""

    def __init__(self, data, rows, cols, kind=Q8_0, device=0):
        self.L = lib()
        self.data = np.ascontiguousarray(data)
        h = C.c_void_p()
        check(self.L.phonon_cuda_linear_create(device, kind, _p(self.data), rows, cols, C.byref(h)),
              "linear_create")
        self.h, self.rows, self.cols = h, rows, cols

    def bytes(self):
        return self.L.phonon_cuda_linear_bytes(self.h)

    def __call__(self, x, bias=None):
        x = np.ascontiguousarray(x, np.float32)
        batch = x.size // self.cols
        y = np.zeros((batch, self.rows), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        check(self.L.phonon_cuda_linear_apply(self.h, _p(x), batch, _p(b), _p(y)), "linear_apply")
        return y

    def apply_device(self, x_ptr, batch, y_ptr, stream_ptr=0, bias_ptr=None, status_ptr=None):
        check(self.L.phonon_cuda_linear_apply_device(self.h, C.c_void_p(x_ptr), batch,
                                                     C.c_void_p(bias_ptr), C.c_void_p(y_ptr),
                                                     C.c_void_p(status_ptr), C.c_void_p(stream_ptr)),
              "linear_apply_device")

    def close(self):
        if self.h:
            self.L.phonon_cuda_linear_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def layer_norm(x, w, b, eps=1e-5, device=0):
    x, w, b = (np.ascontiguousarray(a, np.float32) for a in (x, w, b))
    out = np.zeros_like(x)
    rc = lib().phonon_cuda_layer_norm(device, _p(x), _p(w), _p(b), x.size, eps, _p(out))
    return rc, out


def erf_gelu(x, device=0):
    y = np.array(x, np.float32, copy=True)
    return lib().phonon_cuda_erf_gelu(device, _p(y), y.size), y


def rope(x, heads, position, theta=10000.0, device=0):
    y = np.array(x, np.float32, copy=True)
    return lib().phonon_cuda_rope_interleaved(device, _p(y), y.size, heads, position, theta), y


def i8_gemm(a, b, device=0):
    """D[m][n] = sum_k a[m][k] b[n][k] (int8 in, exact int32 out) on tcgen05."""
    a = np.ascontiguousarray(a, np.int8)
    b = np.ascontiguousarray(b, np.int8)
    m, k = a.shape
    n = b.shape[0]
    d = np.zeros((m, n), np.int32)
    L = lib()
    L.phonon_cuda_i8_gemm.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t,
                                      C.c_size_t, C.c_void_p]
    L.phonon_cuda_i8_gemm.restype = C.c_int
    check(L.phonon_cuda_i8_gemm(device, _p(a), _p(b), m, n, k, _p(d)), "i8_gemm")
    return d


def head_struct(head, frame=None):
    """PhononCudaHeadWeights over a head dict of bf16 arrays (the layout of
    the flow-head tests: (weight, bias) pairs per linear) and, optionally,
    the frame loop's tensors: frame = {"eos": (w [1][512], b [1]),
    "embed": w [512][32], "out_norm": (w, b)}. The arrays must outlive the
    create call."""
    def ptr(a):
        return None if a is None else a.ctypes.data

    def aff(wb):
        return Affine(ptr(wb[0]), ptr(wb[1]))

    w = HeadWeights()
    w.input = aff(head["input"])
    w.cond = aff(head["cond"])
    for t in range(2):
        for j in range(2):
            w.time[t][j] = aff(head["time"][t][j])
        w.time_freqs[t] = ptr(head["time_freqs"][t])
        w.time_alpha[t] = ptr(head["time_alpha"][t])
    for b in range(HEAD_BLOCKS):
        w.block_ada[b] = aff(head["block_ada"][b])
        w.block_norm_w[b] = ptr(head["block_norm_w"][b])
        w.block_norm_b[b] = ptr(head["block_norm_b"][b])
        for j in range(2):
            w.block_mlp[b][j] = aff(head["block_mlp"][b][j])
    w.final_ada = aff(head["final_ada"])
    w.final_out = aff(head["final_out"])
    if frame:
        w.eos = aff(frame["eos"])
        w.embed = ptr(frame["embed"])
        w.out_norm_w = ptr(frame["out_norm"][0])
        w.out_norm_b = ptr(frame["out_norm"][1])
    return w


class Head:
    """A flow head (and the frame loop's tensors) on a context's device."""

    def __init__(self, ctx, head, frame=None):
        self.ctx = ctx
        self.L = lib()
        self._keep = (head, frame)
        w = head_struct(head, frame)
        h = C.c_void_p()
        check(self.L.phonon_cuda_head_create(ctx.h, C.byref(w), C.byref(h)), "head_create")
        self.h = h

    def close(self):
        if self.h:
            self.L.phonon_cuda_head_free(self.h)
            self.h = None

    def set_tensor_min(self, min_batch):
        """Batches of at least min_batch rows take the tensor-core linears;
        returns whether that path is available."""
        ok = C.c_int(0)
        check(self.L.phonon_cuda_head_set_tensor_min(self.h, min_batch, C.byref(ok)), "head_set_tensor_min")
        return bool(ok.value)

    def forward(self, condition, state, s, t):
        condition = np.ascontiguousarray(condition, np.float32).reshape(-1, WIDTH)
        state = np.ascontiguousarray(state, np.float32).reshape(-1, LATENT)
        out = np.zeros((condition.shape[0], LATENT), np.float32)
        check(self.L.phonon_cuda_head_forward(self.h, condition.shape[0], _p(condition), _p(state), s, t, _p(out)),
              "head_forward")
        return out

    def lsd_one_step(self, condition, raw_noise, temperature):
        condition = np.ascontiguousarray(condition, np.float32).reshape(-1, WIDTH)
        raw_noise = np.ascontiguousarray(raw_noise, np.float32).reshape(-1, LATENT)
        out = np.zeros((condition.shape[0], LATENT), np.float32)
        check(self.L.phonon_cuda_lsd_one_step(self.h, condition.shape[0], _p(condition), _p(raw_noise), temperature,
                                              _p(out)), "lsd_one_step")
        return out

    def eos_logit(self, state):
        state = np.ascontiguousarray(state, np.float32).reshape(-1, WIDTH)
        out = np.zeros(state.shape[0], np.float32)
        check(self.L.phonon_cuda_eos_logit(self.h, state.shape[0], _p(state), _p(out)), "eos_logit")
        return out

    def output_norm_device(self, batch, x_ptr, out_ptr):
        check(self.L.phonon_cuda_output_norm_device(self.h, batch, x_ptr, out_ptr), "output_norm_device")

    def frame_step(self, streams, positions, state_ptr, condition_ptr, raw_noise, temperature):
        """One on-device frame; returns (eos logits [n], latents [n][32],
        status [n])."""
        n = len(streams)
        st = np.ascontiguousarray(streams, np.uint32)
        po = np.ascontiguousarray(positions, np.uint32)
        raw_noise = np.ascontiguousarray(raw_noise, np.float32).reshape(n, LATENT)
        logit = np.zeros(n, np.float32)
        latent = np.zeros((n, LATENT), np.float32)
        status = np.zeros(n, np.int32)
        check(self.L.phonon_cuda_frame_step(self.h, n, _p(st), _p(po), state_ptr, condition_ptr, _p(raw_noise),
                                            temperature, _p(logit), _p(latent), _p(status)), "frame_step")
        return logit, latent, status


class Mimi:
    """The Mimi latent transformer on a device: model = {"projection": [512][32],
    "upsample": [512][32], "layers": [{in_proj, out_proj, linear1, linear2,
    norm1_w, norm1_b, norm2_w, norm2_b, scale1, scale2}] * 2} as bf16 arrays."""

    FIELDS = ("in_proj", "out_proj", "linear1", "linear2", "norm1_w", "norm1_b", "norm2_w", "norm2_b",
              "scale1", "scale2")

    def __init__(self, model, device=0, max_states=8, max_batch=8):
        self.L = lib()
        w = MimiWeights()
        w.projection = np.ascontiguousarray(model["projection"]).ctypes.data
        w.upsample = np.ascontiguousarray(model["upsample"]).ctypes.data
        keep = [model]
        for i, layer in enumerate(model["layers"]):
            for f in self.FIELDS:
                a = np.ascontiguousarray(layer[f])
                keep.append(a)
                getattr(w, f)[i] = a.ctypes.data
        h = C.c_void_p()
        check(self.L.phonon_cuda_mimi_create(device, C.byref(w), max_states, max_batch, C.byref(h)), "mimi_create")
        self.h = h

    def close(self):
        if self.h:
            self.L.phonon_cuda_mimi_destroy(self.h)
            self.h = None

    def set_tensor_min(self, min_states):
        ok = C.c_int(0)
        check(self.L.phonon_cuda_mimi_set_tensor_min(self.h, min_states, C.byref(ok)), "mimi_set_tensor_min")
        return bool(ok.value)

    def alloc(self):
        s = C.c_uint32()
        check(self.L.phonon_cuda_mimi_state_alloc(self.h, C.byref(s)), "mimi_state_alloc")
        return s.value

    def reset(self, s):
        check(self.L.phonon_cuda_mimi_state_reset(self.h, s), "mimi_state_reset")

    def free(self, s):
        check(self.L.phonon_cuda_mimi_state_free(self.h, s), "mimi_state_free")

    def positions(self, s):
        n = C.c_uint64()
        check(self.L.phonon_cuda_mimi_positions(self.h, s, C.byref(n)), "mimi_positions")
        return n.value

    def step(self, states, latents):
        """One frame per state: latents [n][32] -> (features [n][16][512], status [n])."""
        n = len(states)
        st = np.ascontiguousarray(states, np.uint32)
        latents = np.ascontiguousarray(latents, np.float32).reshape(n, 32)
        feats = np.zeros((n, 16, WIDTH), np.float32)
        status = np.zeros(n, np.int32)
        check(self.L.phonon_cuda_mimi_step(self.h, n, _p(st), _p(latents), _p(feats), _p(status)), "mimi_step")
        return feats, status

    def process(self, s, latents):
        latents = np.ascontiguousarray(latents, np.float32).reshape(-1, 32)
        feats = np.zeros((latents.shape[0] * 16, WIDTH), np.float32)
        check(self.L.phonon_cuda_mimi_process(self.h, s, _p(latents), latents.shape[0], _p(feats), feats.shape[0]),
              "mimi_process")
        return feats

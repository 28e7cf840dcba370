"""ctypes access to the CPU oracle (TEST INFRASTRUCTURE ONLY).

Two libraries live under oracle/:

* ``liboracle.so``          -- the C restatement of the reference algorithm
                               (phonon_oracle.c + sleef_u10.c);
* ``_ref/libphonon_ref.so`` -- the unmodified speech-mac sources compiled with
                               the shims in oracle/shim (built only where the
                               reference tree exists; the built file travels).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's reference /
cpu_baseline arm may import this module, and only as the checker.
"""
import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libphonon_ref.so"

F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
Q8_BYTES_PER_32 = 34
LINEAR_SHAPES = {"qkv": (1536, 512), "out": (512, 512), "up": (2048, 512), "down": (512, 2048)}


def reference_root():
    """The speech-mac source tree: $PHONON_REFERENCE_ROOT, else a `reference`
    directory beside the repository checkout (it exists only where the oracle
    is built, never on the GPU box)."""
    env = os.environ.get("PHONON_REFERENCE_ROOT")
    return Path(env) if env else HERE.parent.parent / "reference"


def build(ref_root=None):
    """Compile liboracle.so and, when the reference tree exists, _ref/."""
    cmd = f"make -s -C {HERE}"
    if ref_root:
        cmd += f" REF={ref_root}"
    rc = os.system(cmd)
    if rc != 0:
        raise RuntimeError(f"oracle build failed: {cmd}")


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p)


class OracleLinear(C.Structure):
    _fields_ = [("dtype", C.c_int), ("rows", C.c_size_t), ("cols", C.c_size_t), ("data", C.c_void_p)]


class OracleLayer(C.Structure):
    _fields_ = [("qkv", OracleLinear), ("out", OracleLinear), ("up", OracleLinear),
                ("down", OracleLinear), ("norm1_w", C.c_void_p), ("norm1_b", C.c_void_p),
                ("norm2_w", C.c_void_p), ("norm2_b", C.c_void_p)]


class OracleCache(C.Structure):
    _fields_ = [("n_layers", C.c_size_t), ("capacity", C.c_size_t), ("length", C.c_size_t),
                ("keys", C.POINTER(C.c_float)), ("values", C.POINTER(C.c_float)),
                ("kv_bf16", C.c_int)]


class OracleAffine(C.Structure):
    _fields_ = [("w", OracleLinear), ("b", C.c_void_p)]


HEAD_BLOCKS = 6


class OracleFlowHead(C.Structure):
    _fields_ = [("input", OracleAffine), ("cond", OracleAffine), ("time", (OracleAffine * 2) * 2),
                ("time_freqs", C.c_void_p * 2), ("time_alpha", C.c_void_p * 2),
                ("block_ada", OracleAffine * HEAD_BLOCKS), ("block_norm_w", C.c_void_p * HEAD_BLOCKS),
                ("block_norm_b", C.c_void_p * HEAD_BLOCKS), ("block_mlp", (OracleAffine * 2) * HEAD_BLOCKS),
                ("final_ada", OracleAffine), ("final_out", OracleAffine)]


def flow_head_struct(head):
    """OracleFlowHead over a flow head given as bf16 (uint16) arrays:
    {"input", "cond", "final_ada", "final_out": (W [rows, cols], b [rows]),
     "time": [[(W, b)] * 2] * 2, "time_freqs": [128] * 2, "time_alpha": [512] * 2,
     "block_ada": [(W, b)] * 6, "block_norm_w"/"block_norm_b": [512] * 6,
     "block_mlp": [[(W, b)] * 2] * 6}. The arrays must outlive the struct
    (the caller keeps `head`)."""
    def aff(wb):
        w, b = wb
        assert w.dtype == np.uint16 and b.dtype == np.uint16 and w.flags.c_contiguous
        return OracleAffine(OracleLinear(2, w.shape[0], w.shape[1], w.ctypes.data), b.ctypes.data)

    h = OracleFlowHead()
    h.input, h.cond = aff(head["input"]), aff(head["cond"])
    for i in range(2):
        for j in range(2):
            h.time[i][j] = aff(head["time"][i][j])
        h.time_freqs[i] = head["time_freqs"][i].ctypes.data
        h.time_alpha[i] = head["time_alpha"][i].ctypes.data
    for k in range(HEAD_BLOCKS):
        h.block_ada[k] = aff(head["block_ada"][k])
        h.block_norm_w[k] = head["block_norm_w"][k].ctypes.data
        h.block_norm_b[k] = head["block_norm_b"][k].ctypes.data
        for j in range(2):
            h.block_mlp[k][j] = aff(head["block_mlp"][k][j])
    h.final_ada, h.final_out = aff(head["final_ada"]), aff(head["final_out"])
    return h


class OracleMimi(C.Structure):
    _fields_ = [("projection", OracleLinear), ("upsample", C.c_void_p), ("in_proj", OracleLinear * 2),
                ("out_proj", OracleLinear * 2), ("linear1", OracleLinear * 2), ("linear2", OracleLinear * 2),
                ("norm1_w", C.c_void_p * 2), ("norm1_b", C.c_void_p * 2), ("norm2_w", C.c_void_p * 2),
                ("norm2_b", C.c_void_p * 2), ("scale1", C.c_void_p * 2), ("scale2", C.c_void_p * 2),
                ("rope_theta", C.c_float)]


class OracleMimiState(C.Structure):
    _fields_ = [("position", C.c_size_t), ("failed", C.c_int), ("previous", C.c_float * 512),
                ("keys", C.POINTER(C.c_float)), ("values", C.POINTER(C.c_float))]


MIMI_FIELDS = ("in_proj", "out_proj", "linear1", "linear2", "norm1_w", "norm1_b", "norm2_w", "norm2_b",
               "scale1", "scale2")  # the reference's per-layer tensor order (src/phonon_mimi.c:57-66)
MIMI_SHAPES = {"in_proj": (1536, 512), "out_proj": (512, 512), "linear1": (2048, 512), "linear2": (512, 2048)}


def mimi_struct(model):
    """OracleMimi over a Mimi model given as bf16 (uint16) arrays:
    {"projection": [512, 32], "upsample": [512, 32], "layers": [{field: array}] * 2}
    with the fields of MIMI_FIELDS (matrices [rows, cols], vectors [512])."""
    m = OracleMimi()
    m.projection = OracleLinear(2, 512, 32, model["projection"].ctypes.data)
    m.upsample = model["upsample"].ctypes.data
    for i, layer in enumerate(model["layers"]):
        for f, (rows, cols) in MIMI_SHAPES.items():
            assert layer[f].shape == (rows, cols) and layer[f].dtype == np.uint16
            getattr(m, f)[i] = OracleLinear(2, rows, cols, layer[f].ctypes.data)
        for f in MIMI_FIELDS[4:]:
            getattr(m, f)[i] = layer[f].ctypes.data
    m.rope_theta = 10000.0
    return m


def _head_call(fn, head, condition, state, *scalars):
    out = np.zeros(32, np.float32)
    h = flow_head_struct(head)
    ok = fn(C.byref(h), _ptr(np.ascontiguousarray(condition, np.float32)),
            _ptr(np.ascontiguousarray(state, np.float32)), *[C.c_float(v) for v in scalars], _ptr(out))
    return bool(ok), out


class Oracle:
    """The C restatement."""

    def __init__(self, path=ORACLE_SO):
        if not Path(path).exists():
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        L = self.lib = C.CDLL(str(path))
        L.oracle_half_to_float.restype = C.c_float
        L.oracle_half_to_float.argtypes = [C.c_uint16]
        for name in ["oracle_q8_dot", "oracle_q8_matvec", "oracle_linear_batch",
                     "oracle_layer_norm", "oracle_rms_norm", "oracle_erf_gelu",
                     "oracle_rope_interleaved", "oracle_attention", "oracle_cache_init",
                     "oracle_layer_step", "oracle_layer_step_forced", "oracle_stack_step"]:
            getattr(L, name).restype = C.c_int
        L.oracle_q8_dot.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]
        L.oracle_q8_matvec.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p]
        L.oracle_linear_batch.argtypes = [C.POINTER(OracleLinear), C.c_void_p, C.c_size_t,
                                          C.c_void_p, C.c_void_p]
        L.oracle_layer_norm.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_float,
                                        C.c_void_p]
        L.oracle_rms_norm.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_float, C.c_void_p]
        L.oracle_erf_gelu.argtypes = [C.c_void_p, C.c_size_t]
        L.oracle_rope_interleaved.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t,
                                              C.c_float]
        L.oracle_attention.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t,
                                       C.c_void_p]
        L.oracle_cache_init.argtypes = [C.POINTER(OracleCache), C.c_size_t, C.c_size_t]
        L.oracle_cache_destroy.argtypes = [C.POINTER(OracleCache)]
        L.oracle_layer_step.argtypes = [C.POINTER(OracleLayer), C.POINTER(OracleCache), C.c_size_t,
                                        C.c_size_t, C.c_void_p, C.c_float, C.c_void_p]
        L.oracle_layer_step_forced.argtypes = [C.POINTER(OracleLayer), C.POINTER(OracleCache),
                                               C.c_size_t, C.c_size_t, C.c_void_p, C.c_float,
                                               C.c_void_p, C.c_void_p, C.c_void_p]
        L.oracle_stack_step.argtypes = [C.POINTER(OracleLayer), C.c_size_t, C.POINTER(OracleCache),
                                        C.c_size_t, C.c_void_p, C.c_float, C.c_void_p, C.c_void_p]
        L.oracle_flow_head_forward.restype = C.c_int
        L.oracle_flow_head_forward.argtypes = [C.POINTER(OracleFlowHead), C.c_void_p, C.c_void_p,
                                               C.c_float, C.c_float, C.c_void_p]
        L.oracle_flow_lsd_one_step.restype = C.c_int
        L.oracle_flow_lsd_one_step.argtypes = [C.POINTER(OracleFlowHead), C.c_void_p, C.c_void_p,
                                               C.c_float, C.c_void_p]
        L.oracle_mimi_state_init.restype = C.c_int
        L.oracle_mimi_state_init.argtypes = [C.POINTER(OracleMimiState)]
        L.oracle_mimi_state_free.argtypes = [C.POINTER(OracleMimiState)]
        L.oracle_mimi_state_reset.argtypes = [C.POINTER(OracleMimiState)]
        L.oracle_mimi_upsample_frame.restype = C.c_int
        L.oracle_mimi_upsample_frame.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t,
                                                 C.c_void_p]
        L.oracle_mimi_process.restype = C.c_int
        L.oracle_mimi_process.argtypes = [C.POINTER(OracleMimi), C.POINTER(OracleMimiState), C.c_void_p,
                                          C.c_size_t, C.c_void_p]

    # flow head ---------------------------------------------------------------
    def flow_head_forward(self, head, condition, state, s, t):
        """(ok, velocity[32]) of the flow head (see flow_head_struct)."""
        return _head_call(self.lib.oracle_flow_head_forward, head, condition, state, s, t)

    def flow_lsd_one_step(self, head, condition, raw_noise, temperature):
        return _head_call(self.lib.oracle_flow_lsd_one_step, head, condition, raw_noise, temperature)

    # Mimi --------------------------------------------------------------------
    def mimi(self, model):
        return OracleMimiRunner(self, model)

    def mimi_upsample(self, weight, x, previous, channels, stride):
        out = np.zeros(channels * stride, np.float32)
        ok = self.lib.oracle_mimi_upsample_frame(_ptr(weight), _ptr(np.ascontiguousarray(x, np.float32)),
                                                 _ptr(np.ascontiguousarray(previous, np.float32)), channels,
                                                 stride, _ptr(out))
        return bool(ok), out

    # primitives -------------------------------------------------------------
    def half_to_float(self, bits):
        return self.lib.oracle_half_to_float(bits)

    def q8_dot(self, blocks, x):
        out = C.c_float()
        ok = self.lib.oracle_q8_dot(_ptr(blocks), _ptr(x), x.size, C.byref(out))
        return ok, out.value

    def q8_matvec(self, blocks, x, rows, cols, out=None):
        out = np.zeros(rows, np.float32) if out is None else out
        ok = self.lib.oracle_q8_matvec(_ptr(blocks), _ptr(x), rows, cols, _ptr(out))
        return ok, out

    def linear(self, dtype, data, rows, cols, x, batch=1, bias=None):
        lin = OracleLinear(dtype, rows, cols, data.ctypes.data)
        out = np.zeros(batch * rows, np.float32)
        ok = self.lib.oracle_linear_batch(C.byref(lin), _ptr(x), batch,
                                          None if bias is None else _ptr(bias), _ptr(out))
        return ok, out

    def layer_norm(self, x, w, b, eps=1e-5):
        out = np.zeros_like(x)
        ok = self.lib.oracle_layer_norm(_ptr(x), _ptr(w), _ptr(b), x.size, eps, _ptr(out))
        return ok, out

    def rms_norm(self, x, w, eps=1e-5):
        out = np.zeros_like(x)
        ok = self.lib.oracle_rms_norm(_ptr(x), _ptr(w), x.size, eps, _ptr(out))
        return ok, out

    def erf_gelu(self, x):
        y = np.array(x, np.float32, copy=True)
        ok = self.lib.oracle_erf_gelu(_ptr(y), y.size)
        return ok, y

    def rope(self, x, heads, position, theta=10000.0):
        y = np.array(x, np.float32, copy=True)
        ok = self.lib.oracle_rope_interleaved(_ptr(y), y.size, heads, position, theta)
        return ok, y

    def attention(self, q, keys, values, count, stride):
        out = np.zeros(64, np.float32)
        ok = self.lib.oracle_attention(_ptr(q), _ptr(keys), _ptr(values), count, stride, _ptr(out))
        return ok, out

    # model ------------------------------------------------------------------
    def model(self, weights, dtype=1):
        return OracleModel(self, weights, dtype)


class OracleModel:
    """L-layer model over the restatement, one contiguous cache per stream."""

    def __init__(self, oracle, weights, dtype=1):
        self.o = oracle
        self.weights = weights  # keep arrays alive
        self.n_layers = len(weights)
        self.layers = (OracleLayer * self.n_layers)()
        for i, w in enumerate(weights):
            lay = self.layers[i]
            for name in ("qkv", "out", "up", "down"):
                rows, cols = LINEAR_SHAPES[name]
                setattr(lay, name, OracleLinear(dtype, rows, cols, w[name].ctypes.data))
            lay.norm1_w, lay.norm1_b = w["norm1_w"].ctypes.data, w["norm1_b"].ctypes.data
            lay.norm2_w, lay.norm2_b = w["norm2_w"].ctypes.data, w["norm2_b"].ctypes.data

    def new_stream(self, capacity, kv_bf16=False):
        cache = OracleCache()
        if not self.o.lib.oracle_cache_init(C.byref(cache), self.n_layers, capacity):
            raise MemoryError("oracle cache")
        cache.kv_bf16 = 1 if kv_bf16 else 0
        return cache

    def set_kv(self, cache, layer, position, key, value):
        n = cache.capacity * 512
        base = layer * n + position * 512
        keys = np.ctypeslib.as_array(cache.keys, shape=(cache.n_layers * n,))
        vals = np.ctypeslib.as_array(cache.values, shape=(cache.n_layers * n,))
        keys[base:base + 512] = key
        vals[base:base + 512] = value

    def free_stream(self, cache):
        self.o.lib.oracle_cache_destroy(C.byref(cache))

    def step(self, cache, position, x, theta=10000.0, layer_outputs=False):
        out = np.zeros(512, np.float32)
        lo = np.zeros((self.n_layers, 512), np.float32) if layer_outputs else None
        ok = self.o.lib.oracle_stack_step(self.layers, self.n_layers, C.byref(cache), position,
                                          _ptr(np.ascontiguousarray(x, np.float32)), theta,
                                          _ptr(out), None if lo is None else _ptr(lo))
        return ok, out, lo

    def layer_step(self, cache, layer, position, x, theta=10000.0):
        out = np.zeros(512, np.float32)
        ok = self.o.lib.oracle_layer_step(C.byref(self.layers[layer]), C.byref(cache), layer,
                                          position, _ptr(np.ascontiguousarray(x, np.float32)),
                                          theta, _ptr(out))
        return ok, out

    def layer_step_forced(self, cache, layer, position, x, theta=10000.0):
        """Layer step whose K/V row at `position` is the one already in the
        cache (teacher-forced append); returns (ok, y, k, v) with the rows the
        oracle itself computes. Sets cache.length = position first."""
        out = np.zeros(512, np.float32)
        k = np.zeros(512, np.float32)
        v = np.zeros(512, np.float32)
        cache.length = position
        ok = self.o.lib.oracle_layer_step_forced(C.byref(self.layers[layer]), C.byref(cache), layer,
                                                 position, _ptr(np.ascontiguousarray(x, np.float32)),
                                                 theta, _ptr(out), _ptr(k), _ptr(v))
        return ok, out, k, v

    def load_kv(self, cache, keys, values):
        """Rows [0, count) of every layer from keys/values [n_layers][count][512]."""
        n_layers, count = keys.shape[0], keys.shape[1]
        assert n_layers == cache.n_layers and count <= cache.capacity
        shape = (cache.n_layers, cache.capacity, 512)
        ck = np.ctypeslib.as_array(cache.keys, shape=(cache.n_layers * cache.capacity * 512,)).reshape(shape)
        cv = np.ctypeslib.as_array(cache.values, shape=(cache.n_layers * cache.capacity * 512,)).reshape(shape)
        ck[:, :count] = keys
        cv[:, :count] = values

    def kv(self, cache, layer, position):
        n = cache.capacity * 512
        base = layer * n + position * 512
        keys = np.ctypeslib.as_array(cache.keys, shape=(cache.n_layers * n,))
        vals = np.ctypeslib.as_array(cache.values, shape=(cache.n_layers * n,))
        return keys[base:base + 512].copy(), vals[base:base + 512].copy()


class OracleMimiRunner:
    """One request state of the restated Mimi transformer."""

    def __init__(self, oracle, model):
        self.o = oracle
        self.model = model
        self.struct = mimi_struct(model)
        self.state = OracleMimiState()
        if not oracle.lib.oracle_mimi_state_init(C.byref(self.state)):
            raise MemoryError("oracle mimi state")

    def reset(self):
        self.o.lib.oracle_mimi_state_reset(C.byref(self.state))

    def process(self, latents):
        """(ok, features [frames * 16][512]) for latents [frames][32]."""
        latents = np.ascontiguousarray(latents, np.float32).reshape(-1, 32)
        out = np.zeros((latents.shape[0] * 16, 512), np.float32)
        ok = self.o.lib.oracle_mimi_process(C.byref(self.struct), C.byref(self.state), _ptr(latents),
                                            latents.shape[0], _ptr(out))
        return bool(ok), out

    @property
    def position(self):
        return self.state.position

    def close(self):
        self.o.lib.oracle_mimi_state_free(C.byref(self.state))


class PhononMimiConfig(C.Structure):
    """src/phonon_mimi.h:10-16 layout."""
    _fields_ = [("sample_rate", C.c_uint), ("frame_rate", C.c_float), ("ratios", C.c_uint * 3),
                ("context", C.c_size_t), ("rope_theta", C.c_float)]


class PhononTensorView(C.Structure):
    """src/phonon_pack.h:10-19 layout."""
    _fields_ = [("dtype", C.c_int), ("rank", C.c_uint), ("shape", C.c_uint64 * 8),
                ("data", C.c_void_p), ("byte_count", C.c_size_t), ("linear_data", C.c_void_p)]


class PhononMimiModel(C.Structure):
    """src/phonon_mimi.h:19-24 layout."""
    _fields_ = [("config", PhononMimiConfig), ("stride", C.c_size_t), ("projection", PhononTensorView),
                ("upsample", PhononTensorView), ("layers", (PhononTensorView * 10) * 2)]


def _bf16_view(a, shape):
    v = PhononTensorView()
    v.dtype, v.rank = 2, len(shape)
    for i, n in enumerate(shape):
        v.shape[i] = n
    v.data = a.ctypes.data
    v.byte_count = a.size * 2
    return v


class RefMimiRunner:
    """One request state of the reference's own phonon_mimi_process."""

    def __init__(self, ref, model):
        self.r = ref
        self.model = model
        m = self.struct = PhononMimiModel()
        m.config = ref.lib.phonon_mimi_config()
        m.stride = 16
        m.projection = _bf16_view(model["projection"], (512, 32, 1))
        m.upsample = _bf16_view(model["upsample"], (512, 1, 32))
        for i, layer in enumerate(model["layers"]):
            for f_i, f in enumerate(MIMI_FIELDS):
                shape = MIMI_SHAPES[f] if f in MIMI_SHAPES else (512,)
                m.layers[i][f_i] = _bf16_view(layer[f], shape)
        self.state = C.c_void_p()
        if not ref.lib.phonon_mimi_state_create(C.byref(m), C.byref(self.state)):
            raise RuntimeError("phonon_mimi_state_create failed")

    def reset(self):
        self.r.lib.phonon_mimi_state_reset(self.state)

    def process(self, latents):
        latents = np.ascontiguousarray(latents, np.float32).reshape(-1, 32)
        out = np.zeros((latents.shape[0] * 16, 512), np.float32)
        ok = self.r.lib.phonon_mimi_process(self.state, _ptr(latents), latents.shape[0], _ptr(out), out.shape[0])
        return bool(ok), out

    @property
    def position(self):
        return self.r.lib.phonon_mimi_positions(self.state)

    def close(self):
        if self.state:
            self.r.lib.phonon_mimi_state_destroy(self.state)
            self.state = C.c_void_p()


class Reference:
    """The unmodified reference compiled under oracle/_ref."""

    def __init__(self, path=REF_SO, blas_threads=1):
        if not Path(path).exists():
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref`")
        L = self.lib = C.CDLL(str(path))
        L.ref_set_blas_threads.argtypes = [C.c_int]
        L.ref_set_blas_threads(blas_threads)
        L.ref_model_create.restype = C.c_void_p
        L.ref_model_create.argtypes = [C.c_size_t, C.c_int, C.c_void_p, C.c_void_p]
        L.ref_model_destroy.argtypes = [C.c_void_p]
        L.ref_model_prepare.argtypes = [C.c_void_p]
        L.ref_stream_create.restype = C.c_void_p
        L.ref_stream_create.argtypes = [C.c_void_p, C.c_size_t]
        L.ref_stream_destroy.argtypes = [C.c_void_p]
        L.ref_stream_step.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_float,
                                      C.c_void_p, C.c_void_p]
        L.ref_layer_step.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p,
                                     C.c_float, C.c_void_p]
        L.ref_stream_commit.argtypes = [C.c_void_p, C.c_size_t]
        L.ref_stream_prefill.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                         C.c_float, C.c_void_p]
        L.ref_stream_kv.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_void_p]
        L.ref_stream_fill.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_void_p]
        L.ref_stream_length.restype = C.c_size_t
        L.ref_stream_length.argtypes = [C.c_void_p]
        L.ref_flow_head_forward.restype = C.c_int
        L.ref_flow_head_forward.argtypes = [C.POINTER(OracleFlowHead), C.c_void_p, C.c_void_p,
                                            C.c_float, C.c_float, C.c_void_p]
        L.ref_flow_lsd_one_step.restype = C.c_int
        L.ref_flow_lsd_one_step.argtypes = [C.POINTER(OracleFlowHead), C.c_void_p, C.c_void_p,
                                            C.c_float, C.c_void_p]
        L.phonon_q8_dot.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]
        L.phonon_q8_matvec.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p]
        L.phonon_layer_norm.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_float,
                                        C.c_void_p]
        L.phonon_rms_norm.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_float, C.c_void_p]
        L.phonon_erf_gelu.argtypes = [C.c_void_p, C.c_size_t]
        L.phonon_rope_interleaved.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t,
                                              C.c_float]
        L.phonon_attention_test.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                            C.c_size_t, C.c_void_p]
        L.phonon_prefill_attention_test.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p,
                                                    C.c_size_t, C.c_void_p]
        L.phonon_linear_batch.argtypes = [C.POINTER(PhononTensorView), C.c_void_p, C.c_size_t,
                                          C.c_size_t, C.c_void_p, C.c_void_p, C.c_size_t]
        L.phonon_math_sincos.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]
        L.phonon_math_exp4.argtypes = [C.c_void_p]
        L.phonon_math_silu.argtypes = [C.c_void_p, C.c_size_t]
        L.phonon_mimi_config.restype = PhononMimiConfig
        L.phonon_mimi_state_create.restype = C.c_int
        L.phonon_mimi_state_create.argtypes = [C.POINTER(PhononMimiModel), C.POINTER(C.c_void_p)]
        L.phonon_mimi_state_reset.argtypes = [C.c_void_p]
        L.phonon_mimi_state_destroy.argtypes = [C.c_void_p]
        L.phonon_mimi_positions.restype = C.c_size_t
        L.phonon_mimi_positions.argtypes = [C.c_void_p]
        L.phonon_mimi_process.restype = C.c_int
        L.phonon_mimi_process.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]
        L.phonon_mimi_upsample_frame.restype = C.c_int
        L.phonon_mimi_upsample_frame.argtypes = [C.POINTER(PhononTensorView), C.c_void_p, C.c_void_p, C.c_size_t,
                                                 C.c_size_t, C.c_void_p]

    def q8_dot(self, blocks, x):
        out = C.c_float()
        ok = self.lib.phonon_q8_dot(_ptr(blocks), _ptr(x), x.size, C.byref(out))
        return ok, out.value

    def q8_matvec(self, blocks, x, rows, cols, out=None):
        out = np.zeros(rows, np.float32) if out is None else out
        ok = self.lib.phonon_q8_matvec(_ptr(blocks), _ptr(x), rows, cols, _ptr(out))
        return ok, out

    def linear(self, dtype, data, rows, cols, x, batch=1, bias=None):
        v = PhononTensorView()
        v.dtype, v.rank = dtype, 2
        v.shape[0], v.shape[1] = rows, cols
        v.data = data.ctypes.data
        v.byte_count = rows * cols * 2 if dtype == 2 else rows * cols // 32 * 34
        out = np.zeros(batch * rows, np.float32)
        ok = self.lib.phonon_linear_batch(C.byref(v), _ptr(x), rows, cols,
                                          None if bias is None else _ptr(bias), _ptr(out), batch)
        return ok, out

    def layer_norm(self, x, w, b, eps=1e-5):
        out = np.zeros_like(x)
        ok = self.lib.phonon_layer_norm(_ptr(x), _ptr(w), _ptr(b), x.size, eps, _ptr(out))
        return ok, out

    def erf_gelu(self, x):
        y = np.array(x, np.float32, copy=True)
        ok = self.lib.phonon_erf_gelu(_ptr(y), y.size)
        return ok, y

    def rope(self, x, heads, position, theta=10000.0):
        y = np.array(x, np.float32, copy=True)
        ok = self.lib.phonon_rope_interleaved(_ptr(y), y.size, heads, position, theta)
        return ok, y

    def attention(self, q, keys, values, count, stride):
        out = np.zeros(64, np.float32)
        ok = self.lib.phonon_attention_test(_ptr(q), _ptr(keys), _ptr(values), count, stride,
                                            _ptr(out))
        return ok, out

    def sincos(self, x):
        c = np.zeros_like(x)
        s = np.zeros_like(x)
        self.lib.phonon_math_sincos(_ptr(x), x.size, _ptr(c), _ptr(s))
        return c, s

    def model(self, weights, dtype=1, prepare=False):
        m = RefModel(self, weights, dtype)
        if prepare and not self.lib.ref_model_prepare(m.handle):
            raise RuntimeError("ref_model_prepare failed")
        return m


    # flow head ---------------------------------------------------------------
    def flow_head_forward(self, head, condition, state, s, t):
        """(ok, velocity[32]) of the reference's phonon_flow_head_forward."""
        return _head_call(self.lib.ref_flow_head_forward, head, condition, state, s, t)

    def flow_lsd_one_step(self, head, condition, raw_noise, temperature):
        return _head_call(self.lib.ref_flow_lsd_one_step, head, condition, raw_noise, temperature)

    # Mimi --------------------------------------------------------------------
    def mimi(self, model):
        return RefMimiRunner(self, model)

    def mimi_upsample(self, weight, x, previous, channels, stride):
        out = np.zeros(channels * stride, np.float32)
        v = _bf16_view(weight, (channels, 1, 2 * stride))
        ok = self.lib.phonon_mimi_upsample_frame(C.byref(v), _ptr(np.ascontiguousarray(x, np.float32)),
                                                 _ptr(np.ascontiguousarray(previous, np.float32)), channels,
                                                 stride, _ptr(out))
        return bool(ok), out

class RefModel:
    def __init__(self, ref, weights, dtype=1):
        self.r = ref
        self.weights = weights
        self.n_layers = len(weights)
        lin = (C.c_void_p * (4 * self.n_layers))()
        nrm = (C.c_void_p * (4 * self.n_layers))()
        for i, w in enumerate(weights):
            for j, name in enumerate(("qkv", "out", "up", "down")):
                lin[4 * i + j] = w[name].ctypes.data
            for j, name in enumerate(("norm1_w", "norm1_b", "norm2_w", "norm2_b")):
                nrm[4 * i + j] = w[name].ctypes.data
        self.handle = ref.lib.ref_model_create(self.n_layers, dtype, lin, nrm)
        if not self.handle:
            raise RuntimeError("ref_model_create failed")

    def __del__(self):
        if getattr(self, "handle", None):
            self.r.lib.ref_model_destroy(self.handle)
            self.handle = None

    def new_stream(self, capacity):
        s = self.r.lib.ref_stream_create(self.handle, capacity)
        if not s:
            raise MemoryError("ref stream")
        return s

    def free_stream(self, s):
        self.r.lib.ref_stream_destroy(s)

    def step(self, stream, position, x, theta=10000.0, layer_outputs=False):
        out = np.zeros(512, np.float32)
        lo = np.zeros((self.n_layers, 512), np.float32) if layer_outputs else None
        ok = self.r.lib.ref_stream_step(self.handle, stream, position,
                                        _ptr(np.ascontiguousarray(x, np.float32)), theta,
                                        _ptr(out), None if lo is None else _ptr(lo))
        return ok, out, lo

    def layer_step(self, stream, layer, position, x, theta=10000.0):
        out = np.zeros(512, np.float32)
        ok = self.r.lib.ref_layer_step(self.handle, stream, layer, position,
                                       _ptr(np.ascontiguousarray(x, np.float32)), theta, _ptr(out))
        return ok, out

    def commit(self, stream, position):
        return self.r.lib.ref_stream_commit(stream, position)

    def kv(self, stream, layer, position):
        k = np.zeros(512, np.float32)
        v = np.zeros(512, np.float32)
        ok = self.r.lib.ref_stream_kv(stream, layer, position, _ptr(k), _ptr(v))
        assert ok
        return k, v

    def fill(self, stream, length, keys, values):
        return self.r.lib.ref_stream_fill(stream, self.n_layers, length, _ptr(keys), _ptr(values))

    def length(self, stream):
        return self.r.lib.ref_stream_length(stream)

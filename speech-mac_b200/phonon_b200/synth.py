"""Seeded synthetic weights and inputs (ctypes over libphonon_synth.so).

The generator (xoshiro256** seeded by splitmix64, Box-Muller normals) and
the draw rules are documented in csrc/phonon_synth.h. Weights for an L-layer
Flow stack are drawn layer by layer from one generator seeded with `seed`;
stream inputs come from a second generator per stream.
"""
import ctypes as C

import numpy as np

from ._libs import load_synth

SCALE_PER_LINEAR = 0
SCALE_PER_ROW = 1
Q8_SIZES = {"qkv": 1536 * 512 // 32 * 34, "out": 512 * 512 // 32 * 34,
            "up": 2048 * 512 // 32 * 34, "down": 512 * 2048 // 32 * 34}
# Streams draw inputs from seed ^ STREAM_SALT ^ (stream * STREAM_STRIDE).
STREAM_SALT = 0x5354524541_4D31
STREAM_STRIDE = 0x9E3779B97F4A7C15


class Rng(C.Structure):
    _fields_ = [("s", C.c_uint64 * 4), ("has_spare", C.c_int), ("spare", C.c_float)]


def _lib():
    L = load_synth()
    if not getattr(L, "_typed", False):
        L.phonon_rng_seed.argtypes = [C.POINTER(Rng), C.c_uint64]
        L.phonon_rng_next.restype = C.c_uint64
        L.phonon_rng_next.argtypes = [C.POINTER(Rng)]
        L.phonon_rng_normal.argtypes = [C.POINTER(Rng), C.c_void_p, C.c_size_t]
        L.phonon_rng_uniform.argtypes = [C.POINTER(Rng), C.c_float, C.c_float, C.c_void_p,
                                         C.c_size_t]
        L.phonon_float_to_half.restype = C.c_uint16
        L.phonon_float_to_half.argtypes = [C.c_float]
        L.phonon_float_to_bf16.restype = C.c_uint16
        L.phonon_float_to_bf16.argtypes = [C.c_float]
        L.phonon_synth_q8_linear.argtypes = [C.POINTER(Rng), C.c_size_t, C.c_size_t, C.c_int,
                                             C.c_void_p]
        L.phonon_synth_bf16_normal.argtypes = [C.POINTER(Rng), C.c_float, C.c_float, C.c_void_p,
                                               C.c_size_t]
        L.phonon_synth_layer.argtypes = [C.POINTER(Rng), C.c_int] + [C.c_void_p] * 8
        L._typed = True
    return L


class Generator:
    def __init__(self, seed):
        self.rng = Rng()
        _lib().phonon_rng_seed(C.byref(self.rng), seed & (2**64 - 1))

    def next_u64(self):
        return _lib().phonon_rng_next(C.byref(self.rng))

    def normal(self, n):
        out = np.empty(n, np.float32)
        _lib().phonon_rng_normal(C.byref(self.rng), out.ctypes.data, n)
        return out

    def uniform(self, lo, hi, n):
        out = np.empty(n, np.float32)
        _lib().phonon_rng_uniform(C.byref(self.rng), lo, hi, out.ctypes.data, n)
        return out

    def q8_linear(self, rows, cols, scale_mode=SCALE_PER_ROW):
        out = np.empty(rows * cols // 32 * 34, np.uint8)
        _lib().phonon_synth_q8_linear(C.byref(self.rng), rows, cols, scale_mode, out.ctypes.data)
        return out

    def bf16_normal(self, mean, std, n):
        out = np.empty(n, np.uint16)
        _lib().phonon_synth_bf16_normal(C.byref(self.rng), mean, std, out.ctypes.data, n)
        return out


def flow_weights(n_layers, seed=0, scale_mode=SCALE_PER_LINEAR):
    """List of per-layer dicts: qkv/out/up/down Q8_0 blocks (uint8), norm1_w/b
    and norm2_w/b bf16 bits (uint16)."""
    g = Generator(seed)
    L = _lib()
    layers = []
    for _ in range(n_layers):
        w = {k: np.empty(v, np.uint8) for k, v in Q8_SIZES.items()}
        for k in ("norm1_w", "norm1_b", "norm2_w", "norm2_b"):
            w[k] = np.empty(512, np.uint16)
        L.phonon_synth_layer(C.byref(g.rng), scale_mode, w["qkv"].ctypes.data,
                             w["out"].ctypes.data, w["up"].ctypes.data, w["down"].ctypes.data,
                             w["norm1_w"].ctypes.data, w["norm1_b"].ctypes.data,
                             w["norm2_w"].ctypes.data, w["norm2_b"].ctypes.data)
        layers.append(w)
    return layers


def stream_generator(seed, stream):
    return Generator(seed ^ STREAM_SALT ^ ((stream * STREAM_STRIDE) & (2**64 - 1)))


def float_to_half(x):
    return _lib().phonon_float_to_half(x)


def float_to_bf16(x):
    return _lib().phonon_float_to_bf16(x)


def bf16_to_float(bits):
    return (np.asarray(bits, np.uint32) << 16).view(np.float32)


HEAD_BLOCKS = 6  # PHONON_FLOW_HEAD_BLOCKS


def flow_head(seed=0):
    """A random flow head (src/phonon_sampler.c:160-212 shapes) as bf16 bits:
    {"input", "cond", "final_ada", "final_out": (W [rows][cols], b [rows]),
    "time": [[(W, b)] * 2] * 2, "time_freqs": [128] * 2, "time_alpha": [512] * 2,
    "block_ada": [(W, b)] * 6, "block_norm_w"/"block_norm_b": [512] * 6,
    "block_mlp": [[(W, b)] * 2] * 6}. Weights N(0, 1/cols), biases N(0, 0.05^2),
    gains N(1, 0.1^2), time frequencies exp(-9 k / 127)."""
    g = Generator(seed ^ 0x68656164)

    def lin(rows, cols):
        w = g.bf16_normal(0.0, 1.0 / np.sqrt(cols), rows * cols).reshape(rows, cols)
        return np.ascontiguousarray(w), g.bf16_normal(0.0, 0.05, rows)

    freqs = np.array([float_to_bf16(float(np.exp(-9.0 * k / 127))) for k in range(128)], np.uint16)
    return {
        "input": lin(512, 32), "cond": lin(512, 512),
        "time": [[lin(512, 256), lin(512, 512)] for _ in range(2)],
        "time_freqs": [freqs, freqs.copy()],
        "time_alpha": [g.bf16_normal(1.0, 0.1, 512) for _ in range(2)],
        "block_ada": [lin(1536, 512) for _ in range(HEAD_BLOCKS)],
        "block_norm_w": [g.bf16_normal(1.0, 0.1, 512) for _ in range(HEAD_BLOCKS)],
        "block_norm_b": [g.bf16_normal(0.0, 0.1, 512) for _ in range(HEAD_BLOCKS)],
        "block_mlp": [[lin(512, 512), lin(512, 512)] for _ in range(HEAD_BLOCKS)],
        "final_ada": lin(1024, 512), "final_out": lin(32, 512),
    }


def frame_tensors(seed=0):
    """The frame loop's pack tensors next to the head, as bf16 bits:
    flow_lm.out_eos (w [1][512], b [1]), flow_lm.input_linear.weight
    [512][32], flow_lm.out_norm (w, b [512])."""
    g = Generator(seed ^ 0x6672616d)
    return {
        "eos": (g.bf16_normal(0.0, 1.0 / np.sqrt(512), 512).reshape(1, 512), g.bf16_normal(0.0, 0.1, 1)),
        "embed": np.ascontiguousarray(g.bf16_normal(0.0, 1.0 / np.sqrt(32), 512 * 32).reshape(512, 32)),
        "out_norm": (g.bf16_normal(1.0, 0.05, 512), g.bf16_normal(0.0, 0.05, 512)),
    }


def mimi_model(seed=0):
    """A random Mimi latent transformer (src/phonon_mimi.c:47-82 shapes) as
    bf16 bits: {"projection": [512][32], "upsample": [512][32], "layers":
    [{in_proj [1536][512], out_proj [512][512], linear1 [2048][512],
    linear2 [512][2048], norm1_w/b, norm2_w/b, scale1, scale2 [512]}] * 2}.
    Weights N(0, 1/cols), gains N(1, 0.1^2), biases N(0, 0.1^2), layer
    scales N(0.2, 0.05^2)."""
    g = Generator(seed ^ 0x6d696d69)

    def mat(rows, cols):
        return np.ascontiguousarray(g.bf16_normal(0.0, 1.0 / np.sqrt(cols), rows * cols).reshape(rows, cols))

    layers = []
    for _ in range(2):
        layers.append({
            "in_proj": mat(1536, 512), "out_proj": mat(512, 512), "linear1": mat(2048, 512),
            "linear2": mat(512, 2048),
            "norm1_w": g.bf16_normal(1.0, 0.1, 512), "norm1_b": g.bf16_normal(0.0, 0.1, 512),
            "norm2_w": g.bf16_normal(1.0, 0.1, 512), "norm2_b": g.bf16_normal(0.0, 0.1, 512),
            "scale1": g.bf16_normal(0.2, 0.05, 512), "scale2": g.bf16_normal(0.2, 0.05, 512),
        })
    return {"projection": mat(512, 32),
            "upsample": np.ascontiguousarray(g.bf16_normal(0.0, 0.3, 512 * 32).reshape(512, 32)),
            "layers": layers}


def per_block_scales(weights, seed):
    """Copies of Q8_0 layers (flow_weights) whose 32-blocks carry their own
    fp16 scales, as real packs do: each block's scale is the linear's scale
    times U(0.1, 1) (up to 10x apart within a row), and eight blocks per
    linear are zero."""
    rng = np.random.default_rng(seed)
    out = []
    for w in weights:
        w2 = dict(w)
        for k in ("qkv", "out", "up", "down"):
            blob = w[k].copy().reshape(-1, 34)
            base = blob[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
            scale = (base * rng.uniform(0.1, 1.0, blob.shape[0])).astype(np.float16)
            scale[rng.integers(0, blob.shape[0], 8)] = 0.0
            blob[:, 0:2] = scale.view(np.uint8).reshape(-1, 2)
            w2[k] = np.ascontiguousarray(blob.reshape(-1))
        out.append(w2)
    return out

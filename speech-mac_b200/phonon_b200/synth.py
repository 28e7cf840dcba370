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

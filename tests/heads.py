"""Flow heads for the head tests (test helper): the synthetic head of the
reference's sampler test, its inputs, and seeded random heads, all as bf16
(uint16) arrays in the layout of oracle.flow_head_struct."""
import numpy as np

from oracle.oracle import HEAD_BLOCKS

# Chained-output bound, as for the transformer stack: two correct fp32
# evaluations that only order their sums differently (sequential vs SGEMM)
# differ by up to ~1.2e-4 after the six residual blocks on these heads.
REL_TOL = 1e-3


def rel_err(a, r):
    a, r = np.asarray(a, np.float64), np.asarray(r, np.float64)
    floor = 1e-2 * np.abs(r).max()
    return float(np.max(np.abs(a - r) / np.maximum(np.abs(r), floor)))


def bf16_trunc(x):
    """float32 -> bf16 bits by dropping the low half (exact for k / 128)."""
    return (np.asarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_round(x):
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def pinned_head():
    """The synthetic head of tests/test_phonon_sampler.c:148-187: every matrix
    is a window into one bf16 array m[i] = ((5i mod 7) - 3) / 128 starting at a
    small offset; biases, gains, norms and time frequencies follow per-slot
    integer patterns."""
    n = 1536 * 512 + 32
    i = np.arange(n)
    m = bf16_trunc(((i * 5) % 7 - 3) / 128.0)

    def mat(rows, cols, offset):
        return np.ascontiguousarray(m[offset:offset + rows * cols].reshape(rows, cols))

    def vec(count, pattern, kind):
        k = np.arange(count)
        if kind in (1, 2):
            v = 1.0 + (((k * 3 + pattern * 5) % 7) - 3) / 128.0
        elif kind == 3:
            v = (k % 8 + 1) / 128.0
        else:
            v = (((k * 3 + pattern * 5) % 11) - 5) / 128.0
        return bf16_trunc(v)

    def lin(rows, cols, offset, pattern):
        return mat(rows, cols, offset), vec(rows, pattern, 0)

    return {
        "input": lin(512, 32, 1, 1), "cond": lin(512, 512, 2, 2),
        "time": [[lin(512, 256, t + 1, t + 3), lin(512, 512, t + 4, t + 5)] for t in range(2)],
        "time_freqs": [vec(128, 30 + t, 3) for t in range(2)],
        "time_alpha": [vec(512, 32 + t, 2) for t in range(2)],
        "block_ada": [lin(1536, 512, b + 3, b + 4) for b in range(HEAD_BLOCKS)],
        "block_norm_w": [vec(512, 10 + b, 1) for b in range(HEAD_BLOCKS)],
        "block_norm_b": [vec(512, 16 + b, 0) for b in range(HEAD_BLOCKS)],
        "block_mlp": [[lin(512, 512, b + 9, b + 10), lin(512, 512, b + 11, b + 12)]
                      for b in range(HEAD_BLOCKS)],
        "final_ada": lin(1024, 512, 22, 23), "final_out": lin(32, 512, 24, 25),
    }


def pinned_inputs():
    i = np.arange(512)
    condition = (((i * 7) % 13) - 6) / 8.0
    j = np.arange(32)
    state = (((j * 11 + 3) % 17) - 8) / 16.0
    return condition.astype(np.float32), state.astype(np.float32)


def random_head(seed):
    rng = np.random.default_rng(seed)

    def lin(rows, cols):
        w = rng.standard_normal((rows, cols)) / np.sqrt(cols)
        return np.ascontiguousarray(bf16_round(w)), bf16_round(0.05 * rng.standard_normal(rows))

    return {
        "input": lin(512, 32), "cond": lin(512, 512),
        "time": [[lin(512, 256), lin(512, 512)] for _ in range(2)],
        "time_freqs": [bf16_round(np.exp(-np.linspace(0, 9, 128))) for _ in range(2)],
        "time_alpha": [bf16_round(1 + 0.1 * rng.standard_normal(512)) for _ in range(2)],
        "block_ada": [lin(1536, 512) for _ in range(HEAD_BLOCKS)],
        "block_norm_w": [bf16_round(1 + 0.1 * rng.standard_normal(512)) for _ in range(HEAD_BLOCKS)],
        "block_norm_b": [bf16_round(0.1 * rng.standard_normal(512)) for _ in range(HEAD_BLOCKS)],
        "block_mlp": [[lin(512, 512), lin(512, 512)] for _ in range(HEAD_BLOCKS)],
        "final_ada": lin(1024, 512), "final_out": lin(32, 512),
    }




def random_frame(seed):
    """The frame loop's pack tensors around the head (bf16): flow_lm.out_eos
    (w [1][512], b [1]), flow_lm.input_linear.weight [512][32] and
    flow_lm.out_norm (w, b [512])."""
    rng = np.random.default_rng(seed)
    return {
        "eos": (bf16_round(rng.standard_normal((1, 512)) / np.sqrt(512)), bf16_round(0.1 * rng.standard_normal(1))),
        "embed": np.ascontiguousarray(bf16_round(rng.standard_normal((512, 32)) / np.sqrt(32))),
        "out_norm": (bf16_round(1 + 0.05 * rng.standard_normal(512)), bf16_round(0.05 * rng.standard_normal(512))),
    }


def widen(bits):
    """bf16 bits -> float32."""
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)

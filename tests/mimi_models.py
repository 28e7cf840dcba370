"""Mimi latent-transformer models for the Mimi tests (test helper), as bf16
(uint16) arrays in the layout of oracle.mimi_struct: the synthetic model of
the reference's Mimi test with its closed-form expected features, and seeded
random models."""
import numpy as np

from oracle.oracle import MIMI_FIELDS, MIMI_SHAPES

from heads import bf16_round, bf16_trunc


def _empty_layer():
    layer = {f: np.zeros(MIMI_SHAPES[f], np.uint16) for f in MIMI_SHAPES}
    for f in MIMI_FIELDS[4:]:
        layer[f] = np.zeros(512, np.uint16)
    return layer


def synthetic_model():
    """tests/test_phonon_mimi.c:72-94: the projection copies latent element
    i % 32 to channel i, the upsample kernel is 1 for the current frame's
    taps and 0.5 for the previous frame's, Q = K = 0 and V = identity (so
    attention is the plain causal mean over at most 250 rows), out_proj is
    the identity, LayerNorm gains 1, layer scales 0.5 and 0.25, MLP zero."""
    proj = np.zeros((512, 32), np.uint16)
    proj[np.arange(512), np.arange(512) % 32] = bf16_trunc(1.0)
    up = np.zeros((512, 32), np.uint16)
    up[:, :16] = bf16_trunc(1.0)
    up[:, 16:] = bf16_trunc(0.5)
    layers = []
    for li in range(2):
        layer = _empty_layer()
        i = np.arange(512)
        layer["in_proj"][1024 + i, i] = bf16_trunc(1.0)
        layer["out_proj"][i, i] = bf16_trunc(1.0)
        layer["norm1_w"][:] = bf16_trunc(1.0)
        layer["norm2_w"][:] = bf16_trunc(1.0)
        layer["scale1"][:] = bf16_trunc(0.25 if li else 0.5)
        layers.append(layer)
    return {"projection": proj, "upsample": up, "layers": layers}


def synthetic_inputs(frames):
    """input[t][i] = sin((7t + i) * 0.17) in float32 (tests/test_phonon_mimi.c:102-104)."""
    t = np.arange(frames)[:, None]
    i = np.arange(32)[None, :]
    arg = ((t * 7 + i).astype(np.float32) * np.float32(0.17)).astype(np.float32)
    return np.sin(arg).astype(np.float32)


def synthetic_expected(latents):
    """The reference test's independent scalar graph (tests/test_phonon_mimi.c:105-123):
    rows = current latent + 0.5 previous latent, then per layer
    row += scale * causal mean over min(t + 1, 250) LayerNormed rows."""
    frames = latents.shape[0]
    positions = frames * 16
    t = np.arange(positions)
    cur = latents[t // 16][:, np.arange(512) % 32]
    prev = np.where((t >= 16)[:, None], latents[np.maximum(t // 16 - 1, 0)][:, np.arange(512) % 32], 0.0)
    expected = (cur + (np.float32(0.5) * prev).astype(np.float32)).astype(np.float32)
    for li in range(2):
        x = expected.astype(np.float64)
        mean = x.mean(axis=1, keepdims=True)
        var = ((x - mean) ** 2).sum(axis=1, keepdims=True)
        scale = (np.float32(1.0) / np.sqrt((var / 512).astype(np.float32) + np.float32(1e-5))).astype(np.float32)
        norm = ((x - mean).astype(np.float32) * scale).astype(np.float32)
        csum = np.cumsum(norm.astype(np.float64), axis=0)
        out = expected.copy()
        for p in range(positions):
            first = p - 249 if p >= 249 else 0
            s = csum[p] - (csum[first - 1] if first > 0 else 0.0)
            mean_p = (s / (p + 1 - first)).astype(np.float32)
            out[p] = (expected[p] + (np.float32(0.25 if li else 0.5) * mean_p).astype(np.float32)).astype(np.float32)
        expected = out
    return expected


def random_model(seed):
    rng = np.random.default_rng(seed)

    def mat(rows, cols):
        return np.ascontiguousarray(bf16_round(rng.standard_normal((rows, cols)) / np.sqrt(cols)))

    layers = []
    for _ in range(2):
        layer = {f: mat(*MIMI_SHAPES[f]) for f in MIMI_SHAPES}
        layer["norm1_w"] = bf16_round(1 + 0.1 * rng.standard_normal(512))
        layer["norm1_b"] = bf16_round(0.1 * rng.standard_normal(512))
        layer["norm2_w"] = bf16_round(1 + 0.1 * rng.standard_normal(512))
        layer["norm2_b"] = bf16_round(0.1 * rng.standard_normal(512))
        layer["scale1"] = bf16_round(0.2 + 0.05 * rng.standard_normal(512))
        layer["scale2"] = bf16_round(0.2 + 0.05 * rng.standard_normal(512))
        layers.append(layer)
    return {"projection": mat(512, 32), "upsample": np.ascontiguousarray(bf16_round(0.3 * rng.standard_normal((512, 32)))),
            "layers": layers}

"""Small, self-contained workloads of each kernel family, sized for ncu
captures (a few GB on the device at most, a few dozen launches).

    python -m phonon_b200.profile_cases <case>

cases:
  cluster   configs[0]: one stream, 12 layers, fp32 K/V, 128-position
            prefix, 8 single-stream steps (step_cluster_kernel)
  gemv      configs[1]: the four projection shapes at batch 1, eight device
            copies each, one call per copy (gemv_kernel)
  step512   the 512-stream projection chain (two lanes of 256: ln_digits,
            i8_gemm x4, attn_combine_digits, digits<2048>) with short
            contexts (64..128 positions) so the K/V pool stays under 1 GB
  step128   128 streams, contexts U[64, 2048] (seed 2), bf16 K/V
  long8     configs[4]'s late steps: 8 streams at contexts 4000, fp32 K/V,
            per-stage launches (attn_tma_kernel at ~131 MB per launch)
  persist   3 streams at contexts 1000..2000 (step_persist_kernel)
  head512   the flow head at 512 rows on the tensor cores (head_gemm_kernel
            and the head's small kernels), three LSD steps
  frame1    three frames of one stream through phonon_cuda_frame_step
  mimi64    the Mimi latent transformer, 64 states (tensor-core linears),
            rings past the 250-key window, three steps
  perblock512  step512 with per-block-scale Q8_0 weights (three weight
            digit planes on the tensor cores)
Each case runs three steps (or calls) after its set-up and prints "ok".
"""
import sys

import numpy as np

from . import runtime as rt
from . import synth


def _decode(n, lens, kv, steps=3, per_block=False):
    w = synth.flow_weights(12, seed=0)
    if per_block:
        w = synth.per_block_scales(w, 5)
    pages = sum((ln + 8) // 16 + 1 for ln in lens) + 16
    ctx = rt.Context(w, max_streams=n + 2, max_batch=n, pool_pages=pages, kv_type=kv)
    ss = [ctx.stream_alloc(max(lens) + 64) for _ in range(n)]
    for i, (s, ln) in enumerate(zip(ss, lens)):
        ctx.fill_synthetic(s, ln, 77 + i)
    g = synth.Generator(3)
    for t in range(steps):
        ctx.step(ss, [ln + t for ln in lens], g.normal(n * 512).reshape(n, 512))
    ctx.close()


def cluster():
    w = synth.flow_weights(12, seed=0)
    ctx = rt.Context(w, max_streams=2, max_batch=1, pool_pages=32, kv_type=rt.KV_F32)
    assert ctx.set_cluster_step(rt.MAX_POSITIONS), "cluster step unavailable"
    s = ctx.stream_alloc(256)
    g = synth.stream_generator(0, 0)
    ctx.fill_synthetic(s, 128, 5)
    for i in range(8):
        ctx.step([s], [128 + i], g.normal(512)[None])
    ctx.close()


def gemv():
    import torch
    g = synth.Generator(1)
    for rows, cols in ((1536, 512), (512, 512), (2048, 512), (512, 2048)):
        data = g.q8_linear(rows, cols, synth.SCALE_PER_ROW)
        lins = [rt.Linear(data, rows, cols) for _ in range(8)]
        x = torch.randn(1, cols, device="cuda")
        y = torch.empty(1, rows, device="cuda")
        for lin in lins:
            lin.apply_device(x.data_ptr(), 1, y.data_ptr())
        torch.cuda.synchronize()
        for lin in lins:
            lin.close()


def head512():
    w = synth.flow_weights(1, seed=0)
    ctx = rt.Context(w, max_streams=2, max_batch=512, pool_pages=8, kv_type=rt.KV_F32)
    h = rt.Head(ctx, synth.flow_head(0))
    rng = np.random.default_rng(4)
    cond = rng.standard_normal((512, 512)).astype(np.float32)
    for _ in range(3):
        h.lsd_one_step(cond, rng.standard_normal((512, 32)).astype(np.float32), 0.8)
    h.close()
    ctx.close()


def frame1():
    import torch
    w = synth.flow_weights(12, seed=0)
    ctx = rt.Context(w, max_streams=2, max_batch=1, pool_pages=32, kv_type=rt.KV_F32)
    h = rt.Head(ctx, synth.flow_head(0), synth.frame_tensors(0))
    s = ctx.stream_alloc(256)
    ctx.fill_synthetic(s, 128, 5)
    state = torch.randn(1, 512, device="cuda")
    cond = torch.randn(1, 512, device="cuda")
    rng = np.random.default_rng(4)
    for i in range(3):
        _, _, st = h.frame_step([s], [128 + i], state.data_ptr(), cond.data_ptr(),
                                rng.standard_normal((1, 32)).astype(np.float32), 0.8)
        assert not st.any()
    h.close()
    ctx.close()


def mimi64():
    m = rt.Mimi(synth.mimi_model(0), max_states=64, max_batch=64)
    states = [m.alloc() for _ in range(64)]
    rng = np.random.default_rng(5)
    for _ in range(16 + 3):  # 304 positions: past the window
        _, st = m.step(states, rng.standard_normal((64, 32)).astype(np.float32))
        assert not st.any()
    m.close()


CASES = {
    "cluster": cluster,
    "gemv": gemv,
    "step512": lambda: _decode(512, [int(x) for x in np.random.default_rng(2).integers(64, 129, 512)], rt.KV_BF16),
    "step128": lambda: _decode(128, [int(x) for x in np.random.default_rng(2).integers(64, 2049, 128)], rt.KV_BF16),
    "persist": lambda: _decode(3, [1000, 1500, 2000], rt.KV_BF16),
    "long8": lambda: _decode(8, [4000] * 8, rt.KV_F32),
    "head512": head512,
    "frame1": frame1,
    "mimi64": mimi64,
    "perblock512": lambda: _decode(512, [int(x) for x in np.random.default_rng(2).integers(64, 129, 512)], rt.KV_BF16,
                                   per_block=True),
}

if __name__ == "__main__":
    if len(sys.argv) != 2 or sys.argv[1] not in CASES:
        sys.exit(f"usage: python -m phonon_b200.profile_cases {{{'|'.join(CASES)}}}")
    CASES[sys.argv[1]]()
    print("ok")

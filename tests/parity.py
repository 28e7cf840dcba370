"""Teacher-forced per-layer parity of batched decode steps (test helper).

A decode step runs with the context's layer trace on
(phonon_cuda_set_layer_trace), so every layer's output rows of every stream
come back. For a selected stream, the CPU checker is then given exactly what
the device layer saw: the device's own K/V rows (read back bit for bit with
phonon_cuda_kv_read, the row appended at the decoded position included) and
the device's output of the previous layer as input. Its layer output is
compared with the device's, and the K/V row it computes with the device's
appended row. So every layer of the batched step is bounded on its own
(per-layer tolerance), whatever path the step took (per-stage GEMVs,
tensor-core projections, two lanes, ticketed attention, the persistent or the
cluster kernel).

Metrics: rt.rel_err (max_i |a_i - r_i| / max(|r_i|, 1e-2 * max|r|), the bound
of the parity tests) and the normwise error max|a - r| / max|r|.
"""
import numpy as np

from phonon_b200 import runtime as rt

PER_LAYER_TOL = 1e-4


def normwise(a, r):
    a = np.asarray(a, np.float64)
    r = np.asarray(r, np.float64)
    return float(np.max(np.abs(a - r)) / max(np.max(np.abs(r)), 1e-30))


class Trace:
    """Device buffer for the per-layer trace of steps of up to `rows` streams."""

    def __init__(self, ctx, rows):
        import torch
        self.ctx = ctx
        self.rows = rows
        self.buf = torch.zeros((ctx.n_layers, rows, rt.WIDTH), dtype=torch.float32, device=f"cuda:{ctx.device}")
        ctx.set_layer_trace(self.buf.data_ptr(), rows)

    def read(self, n):
        """[n_layers][n][512] of the last step (n = its batch size)."""
        import torch
        torch.cuda.synchronize(self.ctx.device)
        return self.buf[:, :n].cpu().numpy().copy()

    def close(self):
        self.ctx.set_layer_trace(None, 0)


class Stats:
    def __init__(self):
        self.rel = 0.0
        self.norm = 0.0
        self.kv_rel = 0.0
        self.kv_flips = 0
        self.kv_elems = 0
        self.where = None

    def add(self, a, r, where):
        e = rt.rel_err(a, r)
        if e > self.rel:
            self.rel, self.where = e, where
        self.norm = max(self.norm, normwise(a, r))

    def add_kv(self, dev, ref):
        self.kv_rel = max(self.kv_rel, rt.rel_err(dev, ref))
        self.kv_flips += int(np.count_nonzero(dev != ref))
        self.kv_elems += dev.size

    def __str__(self):
        return (f"per-layer max rel err {self.rel:.2e} (at {self.where}), normwise {self.norm:.2e}; "
                f"appended K/V rows: {self.kv_flips}/{self.kv_elems} elements differ, max rel err {self.kv_rel:.2e}")


def check_stream_oracle(ctx, om, stream, positions, inputs, traces, row, stats, kv_bf16, label=""):
    """Teacher-force the oracle through the traced steps of one stream.

    positions[t]: the position decoded at step t; inputs[t]: its input row
    [512]; traces[t]: the trace of step t ([n_layers][n][512]); row: the
    stream's row in those steps' batches. The device cache is read back after
    the last step, so it holds every appended row."""
    last = positions[-1]
    k, v = ctx.kv_read(stream, 0, last + 1)
    cache = om.new_stream(last + 1, kv_bf16=kv_bf16)
    try:
        om.load_kv(cache, k, v)
        for t, pos in enumerate(positions):
            inp = inputs[t]
            for layer in range(ctx.n_layers):
                ok, y, kr, vr = om.layer_step_forced(cache, layer, pos, inp)
                assert ok, (label, t, layer)
                dev = traces[t][layer][row]
                stats.add(dev, y, (label, "step", t, "layer", layer, "pos", pos))
                stats.add_kv(np.concatenate([k[layer, pos], v[layer, pos]]), np.concatenate([kr, vr]))
                inp = dev
    finally:
        om.free_stream(cache)


def check_stream_reference(ctx, rm, stream, positions, inputs, traces, row, stats, label=""):
    """The same against the unmodified reference build (fp32 K/V only): its
    cache holds the device's rows of positions [0, pos), and its own
    phonon_flow_layer_step appends the row at pos."""
    last = positions[-1]
    k, v = ctx.kv_read(stream, 0, last + 1)
    for t, pos in enumerate(positions):
        rs = rm.new_stream(pos + 1)
        try:
            assert rm.fill(rs, pos, np.ascontiguousarray(k[:, :pos]), np.ascontiguousarray(v[:, :pos]))
            inp = inputs[t]
            for layer in range(ctx.n_layers):
                ok, y = rm.layer_step(rs, layer, pos, inp)
                assert ok, (label, t, layer)
                dev = traces[t][layer][row]
                stats.add(dev, y, (label, "ref step", t, "layer", layer, "pos", pos))
                inp = dev
        finally:
            rm.free_stream(rs)

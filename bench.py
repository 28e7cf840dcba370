"""Benchmark of the B200 Flow-transformer decode step (speech-mac configs).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Headline (one JSON line on rank 0): configs[3] -- 512 concurrent streams,
12 layers, contexts U[64,2048] (seed 2), Poisson arrivals and departures
(mean 1 per step, seed 2), bf16 KV in 16-position pages, streams sharded by
request over N GPUs (no collective on the data path; torch.distributed only
synchronises the timing). `value` is decode frames/s of the whole job with
inputs resident in HBM; `e2e` is the same workload through phonon_cuda_step
with host buffers (H2D of x and D2H of y inside every timed step).

Also reported at N=1: configs[0] (one stream, 128-position prefix + 125
steps, L2 flushed between steps) and configs[1] (Q8 matvec GB/s of weight
bytes, cold HBM and hot L2), plus the reference's C path timed on the host
cores (cpu_baseline).

`--impl reference` times the reference's own CPU path (oracle/_ref, the
unmodified speech-mac C compiled with the oracle shims) on the same workload
and prints the same line with "impl": "reference".
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "speech-mac_b200"))
sys.path.insert(0, str(ROOT))

N_LAYERS = 12
STREAMS = 512
METRIC = "decode frames/s (configs[3]: 512 streams, bf16 KV, 12 layers)"
UNIT = "frames/s"
L2_BYTES = 126 * 2**20
HBM_FALLBACK_GBS = 6650.0
# DRAM bytes (read + write) per algorithmic byte of the attention kernel, from
# one ncu capture of the same kernel on the configs[3] shape at 128 streams
# (profiles/attn_tma_kernel_configs3_128streams.md: 293.07 MB of DRAM traffic
# for 286.35 MB of K/V); scaled by each launch's algorithmic bytes to give
# `traffic`.
ATTN_DRAM_PER_ALGO_BYTE = 1.0235


def measured_hbm_gbs():
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


# Useful int8 multiply-adds of the four projections per decoded frame, counted
# as 2 ops each: 12 layers x (1536 + 512 + 2048) x 512 + 512 x 2048 weights.
PROJ_OPS_PER_FRAME = 2 * N_LAYERS * (1536 * 512 + 512 * 512 + 2048 * 512 + 512 * 2048)
BF16_FALLBACK_TFLOPS = 1590.0


def measured_int8_tops():
    """Dense int8 tensor peak: twice the measured dense bf16 GEMM rate (the
    B200 tensor cores run int8 at twice the bf16 rate); the fallback figure
    when no measurement exists."""
    try:
        return 2.0 * float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"]), \
            "2 x measured bf16 dense"
    except Exception:
        return 2.0 * BF16_FALLBACK_TFLOPS, "2 x fallback bf16 dense"


def projection_roofline(prof, frames):
    """The four projection stages of the profiled steps against the int8
    tensor peak: useful ops (PROJ_OPS_PER_FRAME per frame, digit slicing not
    counted) over the time of the qkv, out, up and down classes (on the
    tensor-core path these include the LayerNorm/digit-slicing launches that
    feed the GEMMs). None when the profile has no projection time."""
    ms = sum(prof.get(k, {}).get("ms", 0.0) for k in ("qkv", "out", "up", "down"))
    if ms <= 0.0 or frames <= 0:
        return None
    peak, kind = measured_int8_tops()
    tops = PROJ_OPS_PER_FRAME * frames / (ms * 1e-3) / 1e12
    return {"bound": "tensor", "achieved": round(tops, 1), "peak": round(peak, 1), "unit": "TOPS",
            "frac": round(tops / peak, 4), "peak_source": kind, "ms": round(ms, 3),
            "ops": "useful int8 ops, 2 per multiply-add of the four projections"}


# ------------------------------------------------------------------ workload
class ServingSim:
    """configs[3] arrival process, identical on every rank.

    Start: 512 streams per rank with prefix lengths U[64, 2048]. Each step:
    D ~ Poisson(world) random active streams finish, then A ~ Poisson(world)
    new streams arrive with prefix U[64, 2048]; every active stream decodes
    one position. Streams go to the rank holding the fewest KV pages (ties:
    lowest rank), so each rank serves the configs[3] workload (weak
    scaling)."""

    def __init__(self, world, seed=2, streams=STREAMS, prefix_max=2048):
        self.rng = np.random.default_rng(seed)
        self.rate = float(world)
        self.prefix_max = prefix_max
        max_active = streams + streams // 2
        self.world = world
        self.max_active = max_active
        self.next_id = 0
        self.active = {}  # id -> [rank, position]
        self.pages = [0] * world
        for _ in range(streams):
            self._arrive()

    def _arrive(self):
        prefix = int(self.rng.integers(64, self.prefix_max + 1))
        rank = min(range(self.world), key=lambda r: (self.pages[r], r))
        sid = self.next_id
        self.next_id += 1
        self.active[sid] = [rank, prefix]
        self.pages[rank] += prefix // 16 + 1
        return sid

    def churn(self):
        """Advance one step of arrivals/departures; returns (left, arrived)."""
        left, arrived = [], []
        for _ in range(int(self.rng.poisson(self.rate))):
            if len(self.active) <= 1:
                break
            ids = sorted(self.active)
            sid = ids[int(self.rng.integers(0, len(ids)))]
            rank, pos = self.active.pop(sid)
            self.pages[rank] -= pos // 16 + 1
            left.append(sid)
        for _ in range(int(self.rng.poisson(self.rate))):
            if len(self.active) < self.max_active:
                arrived.append(self._arrive())
        return left, arrived

    def advance(self):
        for v in self.active.values():
            v[1] += 1
            if v[1] % 16 == 0:
                self.pages[v[0]] += 1


class RankServer:
    """This rank's share of the serving simulation on one libphonon_cuda context."""

    def __init__(self, rt, weights, rank, world, device, total_steps, streams, prefix_max=2048):
        self.rt = rt
        self.rank = rank
        self.sim = ServingSim(world, streams=streams, prefix_max=prefix_max)
        per_rank = (self.sim.max_active + world - 1) // world + 8
        cap_positions = prefix_max + total_steps + 32
        pool = per_rank * (cap_positions // 16 + 1)
        self.ctx = rt.Context(weights, device=device, max_streams=per_rank, max_batch=per_rank,
                              pool_pages=pool, kv_type=rt.KV_BF16)
        self.capacity = cap_positions
        self.slot = {}
        for sid, (r, pos) in self.sim.active.items():
            if r == rank:
                self._admit(sid, pos)

    def _admit(self, sid, prefix):
        s = self.ctx.stream_alloc(self.capacity)
        self.ctx.fill_synthetic(s, prefix, 1000003 * sid + 17)
        self.slot[sid] = s

    def churn(self):
        left, arrived = self.sim.churn()
        for sid in left:
            if sid in self.slot:
                self.ctx.stream_free(self.slot.pop(sid))
        for sid in arrived:
            r, pos = self.sim.active[sid]
            if r == self.rank:
                self._admit(sid, pos)

    def batch(self):
        ids = sorted(sid for sid in self.slot)
        return [self.slot[i] for i in ids], [self.sim.active[i][1] for i in ids]


# -------------------------------------------------------------------- clocks
def nvml_sample_loop(nv, device, period_s, out, keep_going):
    """Body of the clock sampler process: the SM clock and the throttle
    reason bits every period_s, one line "monotonic_s sm_mhz bits" each (the
    first line "max <sm max MHz>" says the sampler is ready)."""
    nv.nvmlInit()
    h = nv.nvmlDeviceGetHandleByIndex(device)
    reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
        getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
    out.write(f"max {nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)}\n")
    out.flush()
    while keep_going():
        try:
            out.write(f"{time.monotonic():.6f} {nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)} {reasons(h)}\n")
            out.flush()
        except Exception:
            pass
        time.sleep(period_s)


def clock_sampler_main(argv):
    """Entry of the sampler process (device, period_s, output file): it
    samples until it is terminated, its parent exits, or 15 minutes pass."""
    import pynvml

    device, period, path = int(argv[0]), float(argv[1]), argv[2]
    parent, t_end = os.getppid(), time.monotonic() + 900.0
    with open(path, "w") as out:
        nvml_sample_loop(pynvml, device, period, out,
                         lambda: os.getppid() == parent and time.monotonic() < t_end)


class ClockSampler:
    """SM clock and throttle reasons sampled during a region.

    NVML (nvidia_ml_py) is sampled every 2 ms by a separate process that
    stamps each sample with the monotonic clock, so that even a region of a
    few tens of milliseconds gets samples and the timed loop neither waits
    for an NVML call nor shares the interpreter with a sampling thread;
    without NVML it falls back to `nvidia-smi -lms 100`. Only samples taken
    between __enter__ and __exit__ count."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device, period_s=0.002, extra_path=None):
        self.device = device
        self.period = period_s
        self.extra_path = extra_path  # prepended to the sampler's sys.path (tests: a fake pynvml)
        self.samples = []  # (sm_mhz, max_mhz, reasons set)
        self.proc = None
        self.sampler = None
        self.path = None
        self.thread = None
        self.t0 = self.t1 = 0.0

    def _start_sampler(self):
        import tempfile

        fd, self.path = tempfile.mkstemp(suffix=".clocks")
        os.close(fd)
        paths = [str(ROOT)] + ([str(self.extra_path)] if self.extra_path else [])
        code = ("import sys; sys.path[:0] = sys.argv[1].split(':'); import bench; "
                "bench.clock_sampler_main(sys.argv[2:])")
        self.sampler = subprocess.Popen(
            [sys.executable, "-c", code, ":".join(reversed(paths)), str(self.device), str(self.period), self.path],
            stdin=subprocess.DEVNULL, stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        deadline = time.monotonic() + 30.0
        while time.monotonic() < deadline and self.sampler.poll() is None:
            with open(self.path) as f:
                if f.readline().startswith("max "):
                    return True
            time.sleep(0.01)
        self._stop_sampler()  # no NVML (or it failed): no samples from this process
        os.unlink(self.path)
        return False

    def _stop_sampler(self):
        if self.sampler is not None:
            self.sampler.terminate()
            try:
                self.sampler.wait(timeout=10)
            except subprocess.TimeoutExpired:
                self.sampler.kill()
                self.sampler.wait()

    def _read_samples(self):
        with open(self.path) as f:
            lines = f.read().splitlines()
        os.unlink(self.path)
        max_mhz = float(lines[0].split()[1])
        for line in lines[1:]:
            f = line.split()
            if len(f) != 3:
                continue
            t, sm, bits = float(f[0]), float(f[1]), int(f[2])
            if self.t0 <= t <= self.t1:
                self.samples.append((sm, max_mhz, {k for k, b in self.REASONS.items() if bits & b}))

    def _smi_loop(self):
        for line in self.proc.stdout:
            f = [x.strip() for x in line.split(",")]
            try:
                sm, mx = float(f[0]), float(f[1])
            except (ValueError, IndexError):
                continue
            names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
            self.samples.append((sm, mx, {n for n, v in zip(names, f[3:7]) if v.lower().startswith("active")}))

    def __enter__(self):
        if not self._start_sampler():
            self.sampler = None
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                     "--format=csv,noheader,nounits", "-lms", "100"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.thread = threading.Thread(target=self._smi_loop, daemon=True)
                self.thread.start()
            except OSError:
                self.thread = None
        self.t0 = time.monotonic()
        return self

    def __exit__(self, *exc):
        self.t1 = time.monotonic()
        if self.sampler is not None:
            time.sleep(2 * self.period)  # the sample that closes the region
            self.t1 = time.monotonic()
            self._stop_sampler()
            self._read_samples()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=10)

    def summary(self):
        sm = [x[0] for x in self.samples]
        reasons = set().union(*[x[2] for x in self.samples]) if self.samples else set()
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(x[1] for x in self.samples) if self.samples else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvml, a sampler process every 2 ms" if self.sampler is not None
                else "nvidia-smi, 100 ms" if self.proc is not None else "none (neither NVML nor nvidia-smi)"}


# --------------------------------------------------------------- GPU arm
def run_ours(args):
    import torch

    from phonon_b200 import runtime as rt
    from phonon_b200 import synth

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} needs {args.gpus} ranks (torchrun), got {world}")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        # The data path has no collective: a host-side gloo group only lines
        # the ranks up around the timed regions and reduces their timings.
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def reduce(x, op):
        if not dist:
            return x
        t = torch.tensor([float(x)], dtype=torch.float64)
        dist.all_reduce(t, op=op)
        return float(t.item())

    weights = synth.flow_weights(N_LAYERS, seed=0)
    total_steps = 2 * (args.warmup + args.steps) + min(args.steps, 60) + 8  # timed, profiled, e2e
    server = RankServer(rt, weights, rank, world, local, total_steps, args.streams * world, args.prefix_max)
    ctx = server.ctx
    stream = torch.cuda.ExternalStream(ctx.cuda_stream())
    max_b = server.sim.max_active + 8
    x_dev = torch.randn(max_b, 512, device="cuda", dtype=torch.float32)
    y_dev = torch.empty(max_b, 512, device="cuda", dtype=torch.float32)

    def device_step():
        server.churn()
        streams, pos = server.batch()
        ctx.step_device(streams, pos, x_dev.data_ptr(), y_dev.data_ptr())
        status = ctx.sync(len(streams))
        if status.any():
            raise RuntimeError(f"non-finite status in {int((status != 0).sum())} streams")
        server.sim.advance()
        return len(streams)

    # Step inputs and outputs in page-locked host memory (what an audio
    # front end hands over): the inputs reach the device by DMA every step.
    host_x = torch.from_numpy(synth.Generator(99 + rank).normal(max_b * 512).reshape(max_b, 512)).pin_memory().numpy()
    host_y = torch.empty((max_b, 512), dtype=torch.float32).pin_memory().numpy()
    h2d = d2h = 0

    def host_step():
        nonlocal h2d, d2h
        server.churn()
        streams, pos = server.batch()
        n = len(streams)
        y = ctx.step(streams, pos, host_x[:n], out=host_y[:n])
        h2d += n * 512 * 4
        d2h += y.nbytes + n * 4
        server.sim.advance()
        return n

    def timed(fn, steps, profile=False):
        barrier()
        if profile:
            ctx.profile(True)
        l0 = ctx.launch_count()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        frames = 0
        with ClockSampler(local) as clocks:
            start.record(stream)
            for _ in range(steps):
                frames += fn()
            end.record(stream)
            end.synchronize()
        barrier()
        ms = start.elapsed_time(end)
        prof = ctx.profile_read() if profile else None
        if profile:
            ctx.profile(False)
        return frames, ms, ctx.launch_count() - l0, prof, clocks.summary()

    for _ in range(args.warmup):
        device_step()
    frames, ms, launches, _, clocks = timed(device_step, args.steps)
    tot_frames = reduce(frames, dist.ReduceOp.SUM if dist else None)
    max_ms = reduce(ms, dist.ReduceOp.MAX if dist else None)
    # Per-kernel roofline: a second pass of the same workload with CUDA events
    # around every launch (kept out of `value`: the events add host work). It
    # runs the batch on one lane: on two lanes a kernel shares the GPU with
    # the other half's launches, and its events would time both.
    prof_steps = min(args.steps, 60)
    ctx.set_batch_paths(split_min_batch=1 << 30)
    prof_frames, prof_ms, _, prof, _ = timed(device_step, prof_steps, profile=True)
    ctx.set_batch_paths()
    for _ in range(args.warmup):
        host_step()
    h2d = d2h = 0
    e_frames, e_ms, _, _, _ = timed(host_step, args.steps)
    e_tot = reduce(e_frames, dist.ReduceOp.SUM if dist else None)
    e_max = reduce(e_ms, dist.ReduceOp.MAX if dist else None)

    strong = None
    if world > 1:
        # configs[3] as specified: 512 streams in total, sharded by request
        # over the N GPUs (the per-GPU batch shrinks as N grows).
        ctx.close()
        server = RankServer(rt, weights, rank, world, local, total_steps, args.streams, args.prefix_max)
        ctx = server.ctx
        stream = torch.cuda.ExternalStream(ctx.cuda_stream())
        for _ in range(args.warmup):
            device_step()
        s_frames, s_ms, _, _, _ = timed(device_step, args.steps)
        s_tot = reduce(s_frames, dist.ReduceOp.SUM)
        s_max = reduce(s_ms, dist.ReduceOp.MAX)
        strong = {"value": round(s_tot / (s_max * 1e-3), 1), "unit": UNIT, "scaling": "strong",
                  "streams_total": args.streams, "streams_per_gpu": round(args.streams / world, 1),
                  "ms_per_step": round(s_max / args.steps, 4),
                  "note": "configs[3] as specified: 512 streams in total sharded over the GPUs"}

    extras = {}
    if world == 1 and not args.quick:
        extras["single_stream"] = bench_single_stream(rt, synth, weights, torch)
        extras["prefill"] = bench_prefill(rt, synth, weights, torch)
        lens3 = [int(x) for x in np.random.default_rng(2).integers(64, 2049, 512)]
        extras["mimi"] = bench_mimi(rt, synth, torch)
        # configs[3]'s streams with per-block-scale Q8_0 (real packs' layout): the three-plane tensor-core path
        lens3b = [int(x) for x in np.random.default_rng(2).integers(64, 2049, 512)]
        extras["per_block_scales"] = {
            "workload": "configs[3] streams (512, U[64,2048] seed 2, bf16 K/V, no churn), per-block fp16 scales",
            **decode_run(rt, synth.per_block_scales(weights, 5), torch, lens3b, 20, rt.KV_BF16)}
        extras["frame_loop"] = {
            "configs3": bench_frame_loop(rt, synth, weights, torch, lens3, rt.KV_BF16, 10),
            "configs0": bench_frame_loop(rt, synth, weights, torch, [128], rt.KV_F32, 100),
        }
        extras["q8_matvec"] = bench_q8_matvec(rt, synth, torch, args.matvec_reps)
        extras["config2"] = bench_config2(rt, weights, torch)
        extras["config4"] = bench_config4(rt, weights, torch)

    if rank == 0:
        peak, peak_kind = measured_hbm_gbs()
        dom = max(prof, key=lambda k: prof[k]["ms"])
        d = prof[dom]
        achieved = d["bytes"] / (d["ms"] * 1e-3) / 1e9
        all_bytes = sum(v["bytes"] for v in prof.values())
        traffic = None
        if dom == "attention" and ATTN_DRAM_PER_ALGO_BYTE:
            traffic = round(ATTN_DRAM_PER_ALGO_BYTE * d["bytes"] / max(d["launches"], 1))
        line = {
            "metric": METRIC, "value": round(tot_frames / (max_ms * 1e-3), 1), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(max_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "configs[3]" if (args.streams, args.prefix_max) == (STREAMS, 2048)
                       else f"configs[3] shape, {args.streams} streams, prefix <= {args.prefix_max}",
                       "streams": args.streams, "streams_total": args.streams * world, "layers": N_LAYERS,
                       "context": "prefix U[64,2048] seed 2, synthetic K/V",
                       "arrivals": f"Poisson({world}) arrivals and departures per step, seed 2",
                       "kv": "bf16, 16-position pages", "weights": "Q8_0 int8 + fp16 scales, seed 0",
                       "parallelism": f"request sharding x{world}, {args.streams} streams per GPU",
                       "l2": "per-step KV reads (~13 GB per GPU) far exceed the 126 MB L2"},
            "roofline": {"bound": "hbm", "kernel": dom,
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "traffic": traffic,
                         "measured_over": f"{prof_steps} profiled steps after the timed region, one lane",
                         "algorithmic_bytes_per_launch": round(d["bytes"] / max(d["launches"], 1)),
                         "avg_launch_us": round(d["ms"] * 1e3 / max(d["launches"], 1), 2),
                         "step_achieved_gbs": round(all_bytes / (prof_ms * 1e-3) / 1e9, 1),
                         "kernels": {k: {"ms": round(v["ms"], 3), "launches": v["launches"],
                                         "gbs": round(v["bytes"] / max(v["ms"], 1e-9) * 1e-6, 1)}
                                     for k, v in prof.items() if v["launches"]}},
            "projections": projection_roofline(prof, prof_frames),
            "e2e": {"value": round(e_tot / (e_max * 1e-3), 1), "unit": UNIT,
                    "h2d_bytes_per_step": int(h2d / args.steps),
                    "d2h_bytes_per_step": int(d2h / args.steps)},
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        if strong:
            line["strong"] = strong
        line.update(extras)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
            if not args.quick:
                cpu = cpu_extras()
                line["single_stream"]["cpu_baseline"] = cpu["config0"]
                line["q8_matvec"]["cpu_baseline"] = cpu["q8_matvec"]
                line["config2"]["cpu_baseline"] = cpu["config2"]
                line["config4"]["cpu_baseline"] = cpu["config4"]
                line["frame_loop"]["cpu_baseline_head"] = cpu["flow_head"]
                line["mimi"]["cpu_baseline"] = cpu["mimi"]
        print(json.dumps(line), flush=True)
    ctx.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def l2_flush(torch, buf):
    buf.add_(1.0)


def bench_single_stream(rt, synth, weights, torch):
    """128-position prefix then 125 decode steps of one stream,
    fp32 KV; the L2 is flushed (256 MB read-modify-write) before every timed
    step. Two passes over two streams with the same prefix and inputs:
    device time (the step is enqueued while the flush still runs, so the
    start event fires when the flush ends and the step follows at once) and
    host-inclusive latency (the GPU idle when the start event is recorded,
    so the host's enqueue of the step is inside the timed window)."""
    ctx = rt.Context(weights, max_streams=2, max_batch=1, pool_pages=32, kv_type=rt.KV_F32)
    cluster = ctx.set_cluster_step(rt.MAX_POSITIONS)
    g = synth.stream_generator(0, 0)
    prefix = np.stack([g.normal(512) for _ in range(128)])
    slots = [ctx.stream_alloc(256), ctx.stream_alloc(256)]
    for s in slots:
        ctx.append(s, prefix)
    xs = torch.tensor(np.stack([g.normal(512) for _ in range(125)]), device="cuda")
    x = torch.empty(512, device="cuda")  # fixed input buffer, as an engine's staging buffer
    y = torch.empty(512, device="cuda")
    stream = torch.cuda.ExternalStream(ctx.cuda_stream())
    flush = torch.zeros(64 * 2**20, device="cuda")  # 256 MB

    def run(slot, behind_flush):
        times = []
        for i in range(125):
            x.copy_(xs[i])
            torch.cuda.synchronize()
            if behind_flush:
                with torch.cuda.stream(stream):
                    l2_flush(torch, flush)  # ~80 us of GPU work while the host enqueues the step
            else:
                l2_flush(torch, flush)
                torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            ctx.step_device([slot], [128 + i], x.data_ptr(), y.data_ptr())
            b.record(stream)
            ctx.sync(1)
            times.append(a.elapsed_time(b))
        return times

    times = run(slots[0], True)
    host_times = run(slots[1], False)
    ctx.close()
    total = sum(times)
    # algorithmic HBM bytes: weights, K/V rows read (positions 0..P) and appended, per layer and step
    kv_row = 2 * 512 * 4
    bytes_ = sum(N_LAYERS * (WEIGHT_BYTES_PER_LAYER + (128 + i + 1) * kv_row + kv_row) for i in range(125))
    gbs = bytes_ / (total * 1e-3) / 1e9
    peak, peak_kind = measured_hbm_gbs()
    return {"workload": "configs[0]", "frames_per_s": round(125 / (total * 1e-3), 1),
            "ms_per_step_median": round(statistics.median(times), 4),
            "hbm_gbs": round(gbs, 1), "hbm_frac": round(gbs / peak, 4), "peak_source": peak_kind,
            "timing": "device: CUDA events around the step, enqueued behind the L2 flush",
            "host_inclusive": {"frames_per_s": round(125 / (sum(host_times) * 1e-3), 1),
                               "ms_per_step_median": round(statistics.median(host_times), 4),
                               "timing": "CUDA events, start recorded on an idle GPU: the host's enqueue "
                                         "of the step (Python, C ABI, launch) is inside the window"},
            "path": {2: "16-CTA cluster step, projections on the tensor cores",
                     1: "16-CTA cluster step"}.get(cluster, "per-stage GEMV step"),
            "l2": "flushed before each step"}


WEIGHT_BYTES_PER_LAYER = 3_342_336  # Q8_0 qkv + out + up + down (34-byte blocks of 32)


def bench_prefill(rt, synth, weights, torch, lengths=(128, 2048)):
    """Prefill (phonon_cuda_append, the batched GPU path of
    phonon_flow_stack_prefill_cancel) of one stream: rows [len][512] from
    host memory through all 12 layers into an empty fp32-K/V stream, timed
    end to end on the host (median of 5 after a warm-up). Positions/s, and
    the causal attention's fp32 arithmetic rate (2 flops per multiply-add,
    q.k and p.v over 8 heads x 64 dims for every key a position attends to),
    the work that dominates a long prefill."""
    out = {}
    g = synth.stream_generator(3, 0)
    for n in lengths:
        ctx = rt.Context(weights, max_streams=2, max_batch=1, pool_pages=n // 16 + 8, kv_type=rt.KV_F32)
        rows = np.stack([g.normal(512) for _ in range(n)])
        times = []
        for rep in range(6):
            s = ctx.stream_alloc(n + 1)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            ctx.append(s, rows)
            times.append(time.perf_counter() - t0)
            ctx.stream_free(s)
        ctx.close()
        t = statistics.median(times[1:])
        flops = N_LAYERS * 2 * 2 * 512 * (n * (n + 1) / 2)
        out[f"len{n}"] = {"positions_per_s": round(n / t, 1), "ms": round(t * 1e3, 3),
                          "attention_tflops": round(flops / t / 1e12, 2)}
    return {"workload": "prefill of one stream (configs[0] prefix and a configs[3]-length context)",
            "timing": "host wall clock around phonon_cuda_append (H2D of the rows and D2H of the last output included)",
            **out}


def decode_run(rt, weights, torch, lengths, steps, kv_type, profile_every=0):
    """Decode `steps` frames of len(lengths) streams whose caches start with
    lengths[i] synthetic positions, every stream in every step (device
    buffers, one sync per step, as a serving loop). Returns frames/s, ms per
    step and the step's algorithmic HBM bytes per second (weights + K/V read
    + K/V appended)."""
    R = len(lengths)
    esize = 2 if kv_type == rt.KV_BF16 else 4
    pages = sum((int(n) + steps + 15) // 16 + 1 for n in lengths)
    ctx = rt.Context(weights, max_streams=R + 1, max_batch=R, pool_pages=pages + 8, kv_type=kv_type)
    ss = [ctx.stream_alloc(int(n) + steps + 1) for n in lengths]
    for i, (s, n) in enumerate(zip(ss, lengths)):
        ctx.fill_synthetic(s, int(n), 500 + i)
    x = torch.randn(R, 512, device="cuda")
    y = torch.empty(R, 512, device="cuda")
    stream = torch.cuda.ExternalStream(ctx.cuda_stream())
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    step_bytes = 0.0
    for k in range(steps):
        pos = [int(n) + k for n in lengths]
        ctx.step_device(ss, pos, x.data_ptr(), y.data_ptr())
        if ctx.sync(R).any():
            raise RuntimeError("non-finite step")
        keys = sum(p + 1 for p in pos)
        step_bytes += N_LAYERS * (WEIGHT_BYTES_PER_LAYER + (keys + R) * 2 * 512 * esize)
    b.record(stream)
    b.synchronize()
    ms = a.elapsed_time(b)
    ctx.close()
    return {"frames_per_s": round(R * steps / (ms * 1e-3), 1), "ms_per_step": round(ms / steps, 4),
            "step_gbs": round(step_bytes / (ms * 1e-3) / 1e9, 1)}


def attention_gbs(rt, weights, torch, lengths, steps, kv_type):
    """Attention-only HBM GB/s: the same decode on the per-stage launches with
    per-launch CUDA events (the persistent step has no separate attention
    launch)."""
    R = len(lengths)
    pages = sum((int(n) + steps + 15) // 16 + 1 for n in lengths)
    ctx = rt.Context(weights, max_streams=R + 1, max_batch=R, pool_pages=pages + 8, kv_type=kv_type)
    ctx.set_batch_paths(rt.FUSED_MAX_BATCH + 1, rt.FUSED_MAX_BATCH, 4)
    ss = [ctx.stream_alloc(int(n) + steps + 1) for n in lengths]
    for i, (s, n) in enumerate(zip(ss, lengths)):
        ctx.fill_synthetic(s, int(n), 500 + i)
    x = torch.randn(R, 512, device="cuda")
    y = torch.empty(R, 512, device="cuda")
    ctx.profile(True)
    for k in range(steps):
        ctx.step_device(ss, [int(n) + k for n in lengths], x.data_ptr(), y.data_ptr())
        ctx.sync(R)
    prof = ctx.profile_read()
    ctx.close()
    att = prof["attention"]
    return round(att["bytes"] / (att["ms"] * 1e-3) / 1e9, 1)


def bench_frame_loop(rt, synth, weights, torch, lengths, kv_type, frames, warmup=3):
    """The whole frame loop on the device (phonon_cuda_frame_step: EOS logit,
    flow head LSD step, embedding, 12-layer decode step, output norm) for
    len(lengths) streams, synthetic K/V prefixes and a random head: stream
    frames per second over `frames` frames (host clock around the
    synchronous call, so the H2D of the noise and the D2H of latents and
    logits are inside), and the head's share of the device time from a
    second, profiled run."""
    R = len(lengths)
    total = warmup + frames
    pages = sum((int(n) + 2 * total + 15) // 16 + 1 for n in lengths)
    ctx = rt.Context(weights, max_streams=R + 1, max_batch=R, pool_pages=pages + 8, kv_type=kv_type)
    head = rt.Head(ctx, synth.flow_head(0), synth.frame_tensors(0))
    try:
        ss = [ctx.stream_alloc(int(n) + 2 * total + 1) for n in lengths]
        for i, (s, n) in enumerate(zip(ss, lengths)):
            ctx.fill_synthetic(s, int(n), 500 + i)
        g = torch.Generator(device="cuda").manual_seed(9)
        x = torch.randn(R, 512, device="cuda", generator=g)
        state = torch.empty(R, 512, device="cuda")
        head.output_norm_device(R, x.data_ptr(), state.data_ptr())
        cond = 0.5 * torch.randn(R, 512, device="cuda", generator=g)
        rng = np.random.default_rng(9)
        noise = rng.standard_normal((total, R, 32)).astype(np.float32)
        pos = [int(n) for n in lengths]

        def frame(k):
            _, _, status = head.frame_step(ss, pos, state.data_ptr(), cond.data_ptr(), noise[k], 0.8)
            if status.any():
                raise RuntimeError("frame failed")
            for i in range(R):
                pos[i] += 1

        for k in range(warmup):
            frame(k)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for k in range(warmup, total):
            frame(k)
        dt = time.perf_counter() - t0
        ctx.profile(True)
        for k in range(frames):
            frame(k % total)
        prof = ctx.profile_read()
        ctx.profile(False)
        dev_ms = sum(v["ms"] for v in prof.values())
        return {"streams": R, "frames": frames, "frames_per_s": round(R * frames / dt, 1),
                "ms_per_frame": round(dt / frames * 1e3, 4),
                "head_ms_per_frame": round(prof["head"]["ms"] / frames, 4),
                "head_share_of_device_time": round(prof["head"]["ms"] / dev_ms, 3),
                "head_launches_per_frame": round(prof["head"]["launches"] / frames, 1),
                "timing": "host clock around the synchronous frame call; head share from per-launch CUDA events"}
    finally:
        head.close()
        ctx.close()


def bench_mimi(rt, synth, torch, batches=(1, 64), frames=40, warmup=3):
    """The Mimi latent transformer (phonon_cuda_mimi_step): one latent frame
    -> 16 feature rows for each of n request states per call, host buffers
    (H2D of the latents and D2H of the features inside), host clock around
    the synchronous call; the states' rings fill past the 250-key window."""
    out = {}
    model = synth.mimi_model(0)
    rng = np.random.default_rng(5)
    for n in batches:
        m = rt.Mimi(model, max_states=n, max_batch=n)
        try:
            states = [m.alloc() for _ in range(n)]
            lat = rng.standard_normal((warmup + frames + 16, n, 32)).astype(np.float32)
            for k in range(16 + warmup):  # past the first 250 positions
                m.step(states, lat[k])
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for k in range(frames):
                _, status = m.step(states, lat[16 + warmup + k])
                if status.any():
                    raise RuntimeError("mimi step failed")
            dt = time.perf_counter() - t0
        finally:
            m.close()
        out[f"states{n}"] = {"frames_per_s": round(n * frames / dt, 1), "ms_per_step": round(dt / frames * 1e3, 4),
                             "feature_rows_per_s": round(16 * n * frames / dt, 1)}
    return {"workload": "Mimi latent transformer, random bf16 model, rings past the 250-key window",
            "timing": "host clock around phonon_cuda_mimi_step (latents up, features down)", **out}


def bench_config2(rt, weights, torch):
    """64 streams, prefixes U[32,512] (seed 1), 250 decode steps,
    fp32 KV pages (synthetic K/V for the prefixes)."""
    lengths = np.random.default_rng(1).integers(32, 513, size=64)
    r = decode_run(rt, weights, torch, lengths, 250, rt.KV_F32)
    return {"workload": "configs[2]", **r, "bytes": "weights + K/V read + K/V append per step"}


def bench_config4(rt, weights, torch):
    """8 streams, 256-position prefixes, 4096 decode steps (up to
    4352 positions), fp32 KV; whole-step GB/s over the run and attention-only
    GB/s on a late window (contexts ~4000)."""
    r = decode_run(rt, weights, torch, [256] * 8, 4096, rt.KV_F32)
    att = attention_gbs(rt, weights, torch, [4000] * 8, 40, rt.KV_F32)
    return {"workload": "configs[4]", **r, "attention_gbs_at_4000": att}


def q8_stream_gbs(torch, lins, rows, cols, batch, wbytes, launches):
    """Back-to-back matvecs captured in one CUDA graph (launch overhead out of
    the way, consecutive launches overlapped by programmatic dependent
    launch). Launch i reads lins[i % len(lins)]: with many device copies of
    the matrix, together several times the 126 MB L2, every launch streams
    its weights from HBM; with one copy they stay L2-resident. Returns
    weight GB/s and microseconds per launch."""
    copies = len(lins)
    x = torch.randn(batch, cols, device="cuda")
    y = torch.empty(batch, rows, device="cuda")
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        for lin in lins[:2]:  # first launches configure the kernels outside the capture
            lin.apply_device(x.data_ptr(), batch, y.data_ptr(), side.cuda_stream)
    side.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side, capture_error_mode="relaxed"):
        for i in range(launches):
            lins[i % copies].apply_device(x.data_ptr(), batch, y.data_ptr(), side.cuda_stream)
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    a.record(cur)
    for _ in range(3):
        graph.replay()
    b.record(cur)
    b.synchronize()
    per_launch = a.elapsed_time(b) / (3 * launches)
    del graph
    return round(wbytes / (per_launch * 1e-3) / 1e9, 1), round(per_launch * 1e3, 3)


def bench_q8_matvec(rt, synth, torch, reps):
    """the four projection shapes, per-row scales, batch 1/8/64;
    GB/s of weight bytes. cold: L2 flushed before every single launch
    (latency of one call); hot: back to back on an L2-resident copy;
    stream_hbm / stream_l2: launches back to back in a CUDA graph over
    rotating HBM-cold copies / one L2-resident copy (throughput, see
    q8_stream_gbs)."""
    g = synth.Generator(1)
    flush = torch.zeros(64 * 2**20, device="cuda")
    out = {}
    stream = torch.cuda.current_stream()
    for name, (rows, cols) in {"qkv": (1536, 512), "out": (512, 512), "up": (2048, 512),
                               "down": (512, 2048)}.items():
        data = g.q8_linear(rows, cols, synth.SCALE_PER_ROW)
        lin = rt.Linear(data, rows, cols)
        wbytes = lin.bytes()
        copies = -(-4 * 126 * 2**20 // wbytes)  # 4x L2
        rot = [lin] + [rt.Linear(data, rows, cols) for _ in range(copies - 1)]
        for batch in (1, 8):
            hbm, hbm_us = q8_stream_gbs(torch, rot, rows, cols, batch, wbytes, copies)
            l2, l2_us = q8_stream_gbs(torch, [lin], rows, cols, batch, wbytes, 512)
            out[f"{name}_b{batch}_stream"] = {"stream_hbm_gbs": hbm, "stream_hbm_us": hbm_us,
                                              "stream_l2_gbs": l2, "stream_l2_us": l2_us, "copies": copies}
        for extra in rot[1:]:
            extra.close()
        for batch in (1, 8, 64):
            x = torch.randn(batch, cols, device="cuda")
            y = torch.empty(batch, rows, device="cuda")
            cold = []
            for _ in range(reps):
                l2_flush(torch, flush)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                lin.apply_device(x.data_ptr(), batch, y.data_ptr(), stream.cuda_stream)
                b.record(stream)
                b.synchronize()
                cold.append(a.elapsed_time(b))
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            for _ in range(20):
                lin.apply_device(x.data_ptr(), batch, y.data_ptr(), stream.cuda_stream)
            a.record(stream)
            for _ in range(reps):
                lin.apply_device(x.data_ptr(), batch, y.data_ptr(), stream.cuda_stream)
            b.record(stream)
            b.synchronize()
            hot = a.elapsed_time(b) / reps
            med = statistics.median(cold)
            out[f"{name}_b{batch}"] = {"cold_gbs": round(wbytes / (med * 1e-3) / 1e9, 1),
                                       "hot_gbs": round(wbytes / (hot * 1e-3) / 1e9, 1),
                                       "cold_us": round(med * 1e3, 2), "hot_us": round(hot * 1e3, 2)}
        lin.close()
    return {"workload": "configs[1]", "reps": reps, "weight_bytes": "rows*cols*34/32", **out}


# --------------------------------------------------------------- CPU baseline
def numpy_flow_weights(n_layers, seed=0):
    """Weights of the configs' architecture for the CPU reference runs, drawn
    with numpy (PCG64) in the same distributions as the shared generator:
    Q8_0 blocks with one binary16 scale U(0.5,1.5)/(127*sqrt(cols)) per
    linear and int8 values uniform in [-127, 127]; LayerNorm gamma ~
    N(1, 0.02), beta ~ N(0, 0.02) as bf16. The reference's step time does not
    depend on the values, and this keeps the reference arm free of this
    repository's native code."""
    rng = np.random.default_rng(seed)
    shapes = {"qkv": (1536, 512), "out": (512, 512), "up": (2048, 512), "down": (512, 2048)}

    def bf16(x):
        u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)

    layers = []
    for _ in range(n_layers):
        w = {}
        for name, (rows, cols) in shapes.items():
            scale = np.float16(rng.uniform(0.5, 1.5) / (127.0 * np.sqrt(cols)))
            blocks = np.empty((rows * cols // 32, 34), np.uint8)
            blocks[:, 0:2] = np.frombuffer(scale.tobytes(), np.uint8)
            blocks[:, 2:] = rng.integers(-127, 128, (rows * cols // 32, 32), dtype=np.int8).view(np.uint8)
            w[name] = blocks.ravel()
        for name, mean in (("norm1_w", 1.0), ("norm1_b", 0.0), ("norm2_w", 1.0), ("norm2_b", 0.0)):
            w[name] = bf16(mean + 0.02 * rng.standard_normal(512))
        layers.append(w)
    return layers


class RefRunner:
    """The reference (oracle/_ref) decoding one stream per host thread:
    contexts filled with seeded K/V rows through the public PhononKvCache,
    prepared fp32 linears, OpenBLAS single-threaded per call. Default
    contexts: the configs[3] draw U[64,2048] (seed 2)."""

    def __init__(self, threads, lens=None):
        from oracle.oracle import REF_SO, Reference
        if not REF_SO.exists():
            raise FileNotFoundError("oracle/_ref/libphonon_ref.so is not built")
        self.threads = threads
        ref = Reference(blas_threads=1)
        self.model = ref.model(numpy_flow_weights(N_LAYERS, seed=0), prepare=True)
        rng = np.random.default_rng(2)
        self.lens = [int(x) for x in rng.integers(64, 2049, threads)] if lens is None else list(lens)
        self.cap = max(self.lens) + 2048
        kv = rng.standard_normal((N_LAYERS, max(self.lens), 512), dtype=np.float32)
        self.streams = []
        for t in range(threads):
            s = self.model.new_stream(self.cap)
            keys = np.ascontiguousarray(kv[:, :self.lens[t]])
            self.model.fill(s, self.lens[t], keys, keys)
            self.streams.append(s)
        self.pos = list(self.lens)
        self.x = [np.random.default_rng(5 + t).standard_normal(512).astype(np.float32) for t in range(threads)]

    def run(self, seconds):
        frames = [0] * self.threads
        stop = threading.Event()

        def work(t):
            while not stop.is_set() and self.pos[t] < self.cap:
                ok, _, _ = self.model.step(self.streams[t], self.pos[t], self.x[t])
                if not ok:
                    raise RuntimeError("reference step failed")
                self.pos[t] += 1
                frames[t] += 1

        workers = [threading.Thread(target=work, args=(t,)) for t in range(self.threads)]
        t0 = time.perf_counter()
        for w in workers:
            w.start()
        time.sleep(seconds)
        stop.set()
        for w in workers:
            w.join()
        return sum(frames), time.perf_counter() - t0

    def close(self):
        for s in self.streams:
            self.model.free_stream(s)


def cpu_extras(seconds=3.0):
    """The reference's CPU path on the other configs, on the box's host cores
    (bounded samples, a few seconds each): configs[0] on one thread,
    configs[1] through phonon_q8_matvec on one thread, configs[2] and
    configs[4] with one stream per host thread."""
    out = {}
    threads = cpu_threads()
    r = RefRunner(1, lens=[128])
    r.run(0.5)
    f, dt = r.run(seconds)
    r.close()
    out["config0"] = {"value": round(f / dt, 1), "unit": "frames/s", "cores": 1, "kind": "reference",
                      "sample": f"1 stream, 12 layers, fp32 KV, contexts from 128 on, {f} frames in {dt:.1f} s"}
    from oracle.oracle import Reference
    ref = Reference(blas_threads=1)
    rng = np.random.default_rng(1)
    mv = {}
    for name, (rows, cols) in {"qkv": (1536, 512), "out": (512, 512), "up": (2048, 512),
                               "down": (512, 2048)}.items():
        blocks = np.empty((rows * cols // 32, 34), np.uint8)
        blocks[:, 0:2] = np.frombuffer(np.float16(1.0 / 127).tobytes(), np.uint8)
        blocks[:, 2:] = rng.integers(-127, 128, (rows * cols // 32, 32), dtype=np.int8).view(np.uint8)
        x = rng.standard_normal(cols).astype(np.float32)
        y = np.zeros(rows, np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds / 4:
            ref.q8_matvec(blocks, x, rows, cols, y)
            n += 1
        dt = time.perf_counter() - t0
        mv[name] = round(blocks.nbytes * n / dt / 1e9, 2)
    out["q8_matvec"] = {"gbs": mv, "unit": "GB/s of weight bytes", "cores": 1, "kind": "reference",
                        "sample": f"phonon_q8_matvec, batch 1, {seconds / 4:.2f} s per shape"}
    from phonon_b200 import synth
    head = synth.flow_head(0)
    cond = rng.standard_normal(512).astype(np.float32)
    noise = rng.standard_normal(32).astype(np.float32)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds / 4:
        ok, _ = ref.flow_lsd_one_step(head, cond, noise, 0.8)
        assert ok
        n += 1
    dt = time.perf_counter() - t0
    out["flow_head"] = {"value": round(n / dt, 1), "unit": "head steps/s", "cores": 1, "kind": "reference",
                        "sample": f"phonon_flow_lsd_one_step, one row, {n} calls in {dt:.2f} s"}
    mimi = ref.mimi(synth.mimi_model(0))
    lat = rng.standard_normal((4096, 32)).astype(np.float32)
    mimi.process(lat[:16])  # past the first 250 positions
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds / 4 and n < 4000:
        ok, _ = mimi.process(lat[16 + n:17 + n])
        assert ok
        n += 1
    dt = time.perf_counter() - t0
    mimi.close()
    out["mimi"] = {"value": round(n / dt, 1), "unit": "frames/s", "cores": 1, "kind": "reference",
                   "sample": f"phonon_mimi_process, one state, one frame per call, {n} frames in {dt:.2f} s"}
    lens2 = [int(x) for x in np.random.default_rng(1).integers(32, 513, threads)]
    for key, lens, what in (("config2", lens2, "prefixes U[32,512] seed 1"),
                            ("config4", [2304] * min(threads, 8), "contexts 2304 (mid-run of 256..4352)")):
        r = RefRunner(len(lens), lens=lens)
        r.run(0.5)
        f, dt = r.run(seconds)
        r.close()
        out[key] = {"value": round(f / dt, 1), "unit": "frames/s", "cores": len(lens), "kind": "reference",
                    "sample": f"{len(lens)} streams, one per host thread, {what}, fp32 KV, {f} frames in {dt:.1f} s"}
    return out


def cpu_threads():
    return max(1, min(64, len(os.sched_getaffinity(0))))


def cpu_baseline(seconds):
    threads = cpu_threads()
    r = RefRunner(threads)
    r.run(1.0)
    frames, dt = r.run(seconds)
    r.close()
    return {"value": round(frames / dt, 2), "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": f"{threads} streams (one per host thread), contexts U[64,2048] seed 2 "
                      f"(mean {int(np.mean(r.lens))}), 12 layers, fp32 KV, {frames} frames in "
                      f"{dt:.1f} s, OpenBLAS 1 thread per call"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = cpu_threads()
    per_step = max(0.25, args.cpu_seconds / max(args.steps, 1))
    try:
        r = RefRunner(threads)
    except FileNotFoundError as e:
        print(json.dumps({"impl": "reference", "unavailable": str(e)}))
        return
    for _ in range(args.warmup):
        r.run(per_step / 2)
    t_frames, t_time = 0, 0.0
    for _ in range(args.steps):
        f, dt = r.run(per_step)
        t_frames += f
        t_time += dt
    r.close()
    value = round(t_frames / t_time, 2)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t_time * 1e3 / args.steps, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "configs[3]", "streams": threads, "layers": N_LAYERS,
                       "context": "prefix U[64,2048] seed 2",
                       "kv": "fp32 (the reference has no bf16 KV)",
                       "parallelism": f"{threads} host threads"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                             "sample": f"each step: {threads} threads each decode their own "
                                       f"stream for {per_step:.2f} s"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--quick", action="store_true", help="skip the configs[0]/[1] extras")
    ap.add_argument("--prefix-max", type=int, default=2048,
                    help="upper end of the prefix distribution (2048 = configs[3]; smaller for profiling)")
    ap.add_argument("--streams", type=int, default=STREAMS,
                    help="concurrent streams at start (512 = configs[3]; smaller for profiling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--matvec-reps", type=int, default=2000)
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

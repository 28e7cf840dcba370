"""bench.py's roofline helpers, on CPU: the int8 projection figure the bench
adds to its line must be computed from the profile it is given, and be
absent (not an exception) when a profile has no projection time."""
import sys

import bench


def test_projection_roofline_arithmetic():
    prof = {"qkv": {"ms": 10.0}, "out": {"ms": 5.0}, "up": {"ms": 10.0}, "down": {"ms": 5.0},
            "attention": {"ms": 100.0}}
    frames = 1000
    r = bench.projection_roofline(prof, frames)
    ops = bench.PROJ_OPS_PER_FRAME * frames
    assert bench.PROJ_OPS_PER_FRAME == 2 * 12 * 3_145_728  # the four projections, 12 layers
    assert abs(r["achieved"] - ops / 30e-3 / 1e12) < 0.1  # attention time is not counted
    peak, _ = bench.measured_int8_tops()
    assert abs(r["frac"] - r["achieved"] / peak) < 1e-3 and r["unit"] == "TOPS"


def test_projection_roofline_without_projection_time():
    assert bench.projection_roofline({}, 10) is None
    assert bench.projection_roofline({"attention": {"ms": 3.0}}, 10) is None
    assert bench.projection_roofline({"qkv": {"ms": 1.0}}, 0) is None


def test_clock_sampler_samples_each_step(monkeypatch):
    """The timed loop's per-step poll records clocks even when the sampling
    thread gets no interpreter time (a fake NVML: 1900 of 1965 MHz, power cap)."""
    import types

    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=0, nvmlInit=lambda: None, nvmlDeviceGetHandleByIndex=lambda i: i,
        nvmlDeviceGetMaxClockInfo=lambda h, c: 1965, nvmlDeviceGetClockInfo=lambda h, c: 1900,
        nvmlDeviceGetCurrentClocksEventReasons=lambda h: 0x4)
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench.ClockSampler(0, period_s=3600.0) as clocks:
        for _ in range(3):
            clocks.poll()
    s = clocks.summary()
    assert s["samples"] >= 3 and s["sm_mhz"] == 1900.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]

"""bench.py's roofline helpers and clock sampler, on CPU: the int8
projection figure the bench adds to its line must be computed from the
profile it is given, and be absent (not an exception) when a profile has no
projection time; the clock record comes from a sampler process."""
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


FAKE_NVML = """
NVML_CLOCK_SM = 0
def nvmlInit(): pass
def nvmlDeviceGetHandleByIndex(i): return i
def nvmlDeviceGetMaxClockInfo(h, c): return 1965
def nvmlDeviceGetClockInfo(h, c): return 1900
def nvmlDeviceGetCurrentClocksEventReasons(h): return 0x4
"""


def test_nvml_sample_loop_lines():
    """The sampler process's loop: a ready line with the max clock, then one
    stamped line per sample (a fake NVML: 1900 of 1965 MHz, power cap)."""
    import io
    import types

    ns = {}
    exec(FAKE_NVML, ns)
    fake = types.SimpleNamespace(**{k: v for k, v in ns.items() if not k.startswith("__")})
    out, left = io.StringIO(), [3]

    def keep_going():
        left[0] -= 1
        return left[0] >= 0

    bench.nvml_sample_loop(fake, 0, 0.0, out, keep_going)
    lines = out.getvalue().splitlines()
    assert lines[0] == "max 1965" and len(lines) == 4
    assert all(line.split()[1:] == ["1900", "4"] for line in lines[1:])


def test_clock_sampler_process_records_the_region(tmp_path):
    """The sampler runs as its own process (the timed loop never waits on an
    NVML call): samples inside the region are kept, with the reasons decoded."""
    import time

    (tmp_path / "pynvml.py").write_text(FAKE_NVML)
    with bench.ClockSampler(0, period_s=0.002, extra_path=tmp_path) as clocks:
        assert clocks.sampler is not None and clocks.sampler.poll() is None
        time.sleep(0.05)
    s = clocks.summary()
    assert s["samples"] >= 3 and s["sm_mhz"] == 1900.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"] and s["source"].startswith("nvml")
    assert clocks.sampler.returncode is not None  # stopped


def test_clock_sampler_without_nvml(tmp_path, monkeypatch):
    """An NVML that fails to initialise: the sampler process ends at once,
    its file is removed, and the record says where its samples came from
    (nvidia-smi, or none) instead of claiming NVML."""
    import os
    import tempfile

    (tmp_path / "pynvml.py").write_text("def nvmlInit():\n    raise RuntimeError('no NVML')\n")
    scratch = tmp_path / "tmp"
    scratch.mkdir()
    monkeypatch.setattr(tempfile, "tempdir", str(scratch))  # where the sampler's file goes
    monkeypatch.setenv("PATH", str(tmp_path))  # no nvidia-smi either
    with bench.ClockSampler(0, period_s=0.002, extra_path=tmp_path) as clocks:
        assert clocks.sampler is None
    s = clocks.summary()
    assert s["samples"] == 0 and s["sm_mhz"] is None and s["source"].startswith("none")
    assert os.listdir(scratch) == []

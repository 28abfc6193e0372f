"""bench.py's clock record: samples are kept by their timestamps inside the
timed region, throttle reasons are reported by name, and a region shorter
than the sampling period falls back to the nearest sample (and says so).
No GPU: the sampler's output file is written here."""

import datetime
import os
import tempfile
import time

import bench


def _sampler(lines, start, end):
    c = bench.ClockSampler(0)
    fd, c.path = tempfile.mkstemp(suffix=".csv")
    os.close(fd)
    with open(c.path, "w") as f:
        f.write("\n".join(lines) + "\n")
    c.t_start, c.t_end = start, end
    return c


def _line(t, sm=1965, reasons=("Not Active",) * 4):
    ts = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    return f"{ts}, 0, {sm}, 1965, 500.0, 0x0, " + ", ".join(reasons)


def test_samples_inside_the_region_only():
    t0 = time.time()
    lines = [_line(t0 + 0.05 * k, sm=1000 if k < 2 else 1965) for k in range(10)]
    out = _sampler(lines, t0 + 0.12, t0 + 0.31).summary()
    assert out["samples"] == 4 and out["sm_mhz"] == 1965.0
    assert out["reasons"] == [] and "nearest_sample" not in out


def test_throttle_reasons_are_named():
    t0 = time.time()
    lines = [_line(t0 + 0.05 * k, reasons=("Not Active", "Not Active", "Not Active", "Active"))
             for k in range(4)]
    out = _sampler(lines, t0, t0 + 0.2).summary()
    assert out["reasons"] == ["sw_power_cap"]


def test_a_short_region_takes_the_nearest_sample():
    t0 = time.time()
    lines = [_line(t0 + 0.05 * k) for k in range(4)]
    out = _sampler(lines, t0 + 0.051, t0 + 0.06).summary()
    assert out["samples"] == 1 and out["nearest_sample"] is True


def test_no_samples_gives_none():
    t0 = time.time()
    assert _sampler([], t0, t0 + 1).summary() is None

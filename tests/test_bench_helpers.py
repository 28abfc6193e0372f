"""bench.py's host-side helpers on the CPU: the figures it takes from the
committed ncu summary (DRAM traffic and issue-slot occupancy of the dominant
kernel, for the default workload only)."""

import importlib.util
import re
import types
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_profile_figures_for_the_default_workload():
    b = _bench()
    args = types.SimpleNamespace(n_gaussians=1_000_000, width=800, height=800)
    text = (ROOT / "profiles" / "raster_cfg3_1view.md").read_text()
    for kernel in ("raster_bwd", "raster_fwd"):
        traffic, src = b.profiled_traffic(kernel, args)
        want = re.search(rf"<!-- traffic_bytes_per_launch {kernel} (\d+) -->", text)
        assert traffic == int(want.group(1)) and "profiles/" in src
        issue, _ = b.profiled_issue(kernel, args)
        assert 0.0 < issue <= 1.0
    # no capture of other kernels, nor of other workload sizes
    assert b.profiled_issue("loss", args)[0] is None
    small = types.SimpleNamespace(n_gaussians=10, width=800, height=800)
    assert b.profiled_traffic("raster_bwd", small)[0] is None
    assert b.profiled_issue("raster_bwd", small)[0] is None

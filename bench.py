"""Benchmark: train steps/s of the metal-gauss training hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (BASELINE.json's metric is quoted on it, configs[2]): 1M Gaussians
near the surfaces of 20 random ellipsoids, SH degree 3, 800x800, cameras on a
radius-4 hemisphere; one step = a batch of 8 views (sharded over the N GPUs)
rendered, lossed (0.8 L1 + 0.2 (1 - SSIM) against seeded U[0,1] targets) and
back-propagated, then selective Adam on the union-visible Gaussians; with N > 1
the optimizer is sharded (ZeRO-1: the gradient is reduce-scattered over NCCL,
each rank updates its chunk, the parameters are all-gathered). Inputs are
seeded synthetic data of those shapes; the reference's datasets are not
available here.

`value` is whole-job steps/s with every input resident in HBM (K steps timed
with CUDA events, max over ranks). `e2e` is the same metric through the public
API (engine.Trainer.train_step) with the targets copied host->device from
pinned memory every step and the loss read back every step. `--impl
reference` times the reference's algorithm on the host cores (the CPU oracle,
all threads) on the same workload: every view of each timed step, then one
selective Adam update on the views' union visibility.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = ("train steps/s (fwd+bwd+Adam) at 800×800, 1M Gaussians, 1/2/4/8 B200; "
          "% HBM roofline")
WORKLOAD = ("cfg3: 1M Gaussians near the surfaces of 20 random ellipsoids, SH3, 800x800, "
            "100 hemisphere cameras, batch of 8 views per step sharded over the GPUs, "
            "selective Adam on union-visible Gaussians; on several GPUs ZeRO-1 (NCCL "
            "reduce-scatter of the gradient, Adam on each rank's chunk, all-gather of the "
            "parameters)")
# why the reference's own CPU renderer (metal_gauss.torch_ref) is not timed
# beside the oracle: it cannot be installed in this environment
TORCH_REF_UNAVAILABLE = ("the reference package does not install here: its build backend "
                         "(hatchling) is not in the offline wheelhouse, so metal_gauss.torch_ref "
                         "is not importable on the GPU box")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--n-gaussians", type=int, default=1_000_000)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--width", type=int, default=800)
    ap.add_argument("--height", type=int, default=800)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--dense-adam", action="store_true")
    ap.add_argument("--cpu-budget-s", type=float, default=240.0,
                    help="--impl reference: stop timing further steps once this many seconds "
                         "of CPU work have been spent (the line reports the steps run)")
    ap.add_argument("--render", action="store_true",
                    help="forward-only render throughput on cfg4 (3M heavy-tailed Gaussians, "
                         "1920x1080, antialias, 256 orbit views) instead of the training step")
    ap.add_argument("--cfg5-shard", action="store_true",
                    help="cfg5 as one GPU's shard: 6M Gaussians in a 20x20x5 box with a dense "
                         "ground layer, 1600x1200, 8 of the batch's 64 orbit views per step (the "
                         "share of one of 8 GPUs), fused SSIM loss, dense fused Adam over the "
                         "split SH layout; reports peak device memory")
    args = ap.parse_args()
    if args.cfg5_shard:
        args.n_gaussians, args.width, args.height = 6_000_000, 1600, 1200
        args.batch, args.dense_adam = 8 * max(1, args.gpus), True
    return args


# ------------------------------------------------------------------ helpers

def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_ranks(x: float, world: int) -> list[float]:
    """x from every rank, in rank order (all ranks call it)."""
    if world == 1:
        return [x]
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return dict(json.loads(p.read_text()), source="measured")
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 50 ms around the
    timed region. The sampler is running (its first sample written) before
    the region starts; the summary keeps the samples whose timestamps fall
    inside the region, or the one nearest to it when the region is shorter
    than the sampling period."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.t_start = self.t_end = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            deadline = time.time() + 5.0   # until the first sample is written
            while time.time() < deadline and Path(self.path).stat().st_size == 0:
                time.sleep(0.02)
        except (OSError, FileNotFoundError):
            self.proc = None
        self.t_start = time.time()
        return self

    def __exit__(self, *exc):
        self.t_end = time.time()
        if self.proc is not None:
            time.sleep(0.06)   # one more sample after the region
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        if self.path is None or not os.path.exists(self.path):
            return None
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append(dict(ts=ts, sm=float(parts[2]), sm_max=float(parts[3]),
                                 power=float(parts[4]), hw=parts[6], hw_th=parts[7],
                                 sw_th=parts[8], sw_pc=parts[9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        inside = [r for r in rows if self.t_start <= r["ts"] <= self.t_end]
        nearest = not inside
        if nearest:
            mid = 0.5 * (self.t_start + self.t_end)
            inside = [min(rows, key=lambda r: abs(r["ts"] - mid))]
        reasons = set()
        for r in inside:
            for key, name in (("hw", "hw_slowdown"), ("hw_th", "hw_thermal_slowdown"),
                              ("sw_th", "sw_thermal_slowdown"), ("sw_pc", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        out = {"sm_mhz": statistics.median(r["sm"] for r in inside),
               "sm_max_mhz": max(r["sm_max"] for r in inside),
               "power_w_max": max(r["power"] for r in inside),
               "samples": len(inside), "reasons": sorted(reasons),
               "window_s": round(self.t_end - self.t_start, 3)}
        if nearest:
            out["nearest_sample"] = True   # the region was shorter than the 50 ms period
        return out


# ---------------------------------------------------------------- workload

CFG5_METRIC = ("train steps/s (fwd+bwd+fused Adam) of one GPU's cfg5 shard: 6M Gaussians, "
               "1600x1200, 8 views per GPU of a 64-view batch")
CFG5_WORKLOAD = ("cfg5: 6M Gaussians uniform in a 20x20x5 box plus a dense near-ground layer, SH3, "
                 "1600x1200, 64 orbit cameras, 8 views per GPU per step (one GPU's share of a "
                 "64-view batch over 8 GPUs), fused SSIM loss, dense fused Adam over the split SH "
                 "layout")


def workload(args):
    from metal_gauss_b200 import scenes
    if args.cfg5_shard:
        p, views, spec = scenes.config("cfg5", seed=0)
        g = torch.Generator().manual_seed(1234)
        targets_u8 = [torch.randint(0, 256, (v.height, v.width, 3), dtype=torch.uint8,
                                    generator=g) for v in views]
        return p, views, spec, targets_u8
    p, views, spec = scenes.config("cfg3", n=args.n_gaussians, seed=0)
    if args.width != 800 or args.height != 800:
        views = scenes.sphere_views(100, 4.0, args.width, args.height, 40.0, 1, hemisphere=True)
    g = torch.Generator().manual_seed(1234)
    targets_u8 = [torch.randint(0, 256, (v.height, v.width, 3), dtype=torch.uint8, generator=g)
                  for v in views]
    return p, views, spec, targets_u8


from metal_gauss_b200.dp import batch_indices, shard  # noqa: E402


# ---------------------------------------------------------- algorithmic bytes

def stage_bytes(stage: str, n: int, walked: float, P: int, n_tiles: int,
                n_vis: float, views: int = 1) -> float:
    """Compulsory HBM bytes of one launch of a stage, from the dataflow:
    every input read once, every output written once. Raster, pack and loss
    launches are per view; the two preprocess stages are one launch for the
    `views` views of a step. The rasteriser only touches the list entries it
    walks (each tile's list up to its largest stop index), so those -- not all
    pairs -- are counted."""
    if stage == "raster_bwd":
        # per walked entry: id (4) + the 48-byte splat record; per pixel: T,
        # stop, alpha, rgb, dL/drgb (36); per visible Gaussian: its 48-byte
        # gradient record
        return 52.0 * walked + 36.0 * P + 48.0 * n_vis
    if stage == "raster_fwd":
        # per walked entry 52; per tile offsets + order + walk (12); per pixel
        # rgb, alpha, T, stop out (24)
        return 52.0 * walked + 12.0 * n_tiles + 24.0 * P
    if stage == "pack":
        # uv, conic, opacity, colour in; the 48-byte record out; the view's
        # 48-byte gradient record zeroed
        return (36.0 + 48.0 + 48.0) * n
    if stage == "preprocess_fwd":
        # parameters (log-scales and logits for the step prologue) + SH rows
        # once; activations written (16), the 11 accumulated gradient floats
        # zeroed (44), the visibility count written (4); 48 B of outputs per
        # view
        return (44.0 + 192.0 + 16.0 + 44.0 + 4.0) * n + 48.0 * views * n
    if stage == "preprocess_bwd":
        # parameters once; per view gradient record, valid, colour, gated
        # colour gradient; one read-modify-write of 11 gradient floats
        return 44.0 * n + 76.0 * views * n + 88.0 * n
    if stage == "loss":
        # compulsory: the rendered image in (12), the uint8 target in (3), the
        # image gradient out (12); the two tiled kernels' adjoint maps stay
        # out of the count (they are this implementation's intermediate)
        return 27.0 * P
    if stage == "adam":
        return 28.0 * 59 * n + 8.0 * n
    return 0.0


TRAFFIC_PROFILE = ROOT / "profiles" / "raster_cfg3_1view.md"


def profiled_traffic(kernel: str, args):
    """DRAM bytes (read + write) per launch of `kernel`, from the committed
    ncu capture of one view of the default workload, or (None, reason) when
    this run is not that workload or the capture has no figure for it."""
    if (args.n_gaussians, args.width, args.height) != (1_000_000, 800, 800):
        return None, "no capture for this workload size"
    try:
        text = TRAFFIC_PROFILE.read_text()
    except OSError:
        return None, "capture summary missing"
    commit = re.search(r"<!-- capture_commit (\S+) -->", text)
    at = f", captured at commit {commit.group(1)}" if commit else ""
    for name, val in re.findall(r"<!-- traffic_bytes_per_launch (\S+) (\d+) -->", text):
        if name == kernel:
            return int(val), f"{TRAFFIC_PROFILE.relative_to(ROOT)} (ncu --set full, one view{at})"
    return None, f"no capture of {kernel}"


def profiled_issue(kernel: str, args):
    """Share of issue slots busy (per active cycle) of `kernel` in the same
    committed capture, the bound that applies to an issue-limited kernel, or
    (None, reason) as profiled_traffic."""
    if (args.n_gaussians, args.width, args.height) != (1_000_000, 800, 800):
        return None, "no capture for this workload size"
    try:
        text = TRAFFIC_PROFILE.read_text()
    except OSError:
        return None, "capture summary missing"
    for name, val in re.findall(r"<!-- issue_active_pct (\S+) ([0-9.]+) -->", text):
        if name == kernel:
            return round(float(val) / 100.0, 4), \
                f"{TRAFFIC_PROFILE.relative_to(ROOT)} (ncu --set full, one view)"
    return None, f"no capture of {kernel}"


# ---------------------------------------------------------------- our arm

def run_ours(args, rank, world, local):
    from metal_gauss_b200 import _lib
    from metal_gauss_b200.engine import Trainer

    dev = torch.device("cuda", local)
    p, views, spec, targets_u8 = workload(args)
    trainer = Trainer(p, dev, sh_degree=3, background=spec["background"],
                      selective=not args.dense_adam)
    # the images stay bytes on the device; the loss reads them as x / 255
    targets = [t.to(dev) for t in targets_u8]
    B = args.batch
    if B % world:
        raise SystemExit(f"batch {B} is not divisible by {world} GPUs")

    def step(i):
        idx = shard(batch_indices(i, B, len(views)), rank, world)
        return trainer.train_step([views[j] for j in idx], [targets[j] for j in idx], B)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    # instrumented pass: per-stage CUDA events on every stage (its host
    # overhead would perturb the timed region, so it runs separately)
    n_instr = max(2, min(5, args.steps))
    trainer.stage_events = {}
    trainer.walked = []
    for i in range(n_instr):
        step(args.warmup + i)
    torch.cuda.synchronize()
    stage_ms = {k: v for k, v in trainer.stage_times_ms().items()}
    # list entries the rasteriser walks per view, averaged over the
    # instrumented pass's views (the timed steps launch no reduction for it)
    walked = float(torch.stack(trainer.walked).double().mean()) if trainer.walked else 0.0
    # ZeRO-1 on several GPUs: per step, max over ranks, the time the step's
    # stream waited for the counts, loss and geometry reduce-scatter, and at
    # the next step for the geometry and SH all-gathers -- the part of the
    # exchange the overlap does not hide
    coll = {}
    if world > 1:
        waits = ("exchange_wait", "wait_geo_gather", "wait_sh_gather", "allreduce")
        for k in waits:
            v = float(np.sum(stage_ms[k])) / n_instr if k in stage_ms else 0.0
            coll[k + "_ms"] = round(max_over_ranks(v, world), 4)
        # each rank's own stage time per step (its views' kernels, no waits):
        # the spread is the part of exchange_wait that is waiting for the
        # slowest rank rather than for the transfer
        busy = sum(float(np.sum(v)) for k, v in stage_ms.items() if k not in waits) / n_instr
        coll["rank_busy_ms"] = [round(b, 3) for b in gather_ranks(busy, world)]
        # the wait that exposes the most of the exchange, by name
        names = {"exchange_wait_ms": "count/loss all-reduce + geometry reduce-scatter",
                 "wait_geo_gather_ms": "geometry all-gather",
                 "wait_sh_gather_ms": "SH reduce-scatter + all-gather",
                 "allreduce_ms": "gradient all-reduce (replicated optimizer)"}
        top = max(names, key=lambda k: coll.get(k, 0.0))
        coll["limiting"] = names[top]
    singles = {k: v for k, v in stage_ms.items()
               if k in ("raster_bwd", "raster_fwd", "preprocess_fwd", "preprocess_bwd", "loss",
                        "adam")}
    dom = max(singles, key=lambda k: sum(singles[k]))
    # timed region: events only around the dominant kernel
    trainer.stage_events = {}
    trainer.timed_stages = {dom}
    barrier(world)
    L = _lib.load()
    launches0 = L.mg_launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    first = args.warmup + n_instr
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        barrier(world)
        t0.record()
        for i in range(args.steps):
            step(first + i)
        trainer.synchronize_params()   # the last step's parameter gathers, if in flight
        t1.record()
        torch.cuda.synchronize()
        barrier(world)
    launches = L.mg_launch_count() - launches0
    dom_times = trainer.stage_times_ms().get(dom, [])
    trainer.stage_events = None
    trainer.timed_stages = None
    trainer.walked = []
    # visible Gaussians per view: the mean over the last step's views of the
    # projection's valid flags (each view's own visible set)
    V_rank = max(1, len(trainer.last_stats))
    n_vis_view = float(trainer._batch.valid[:V_rank].ne(0).sum()) / V_rank
    # the device error word after the timed steps: 0 unless a bounded wait
    # gave up or an index was out of range, which voids the run
    dev_err = _lib.device_error()
    ms = t0.elapsed_time(t1) / args.steps
    ms = max_over_ranks(ms, world)
    pairs = [s.pairs for s in trainer.last_stats]
    loss_val = float(trainer.loss.item())

    # roofline of the dominant single-kernel stage, timed live in the timed region
    P = args.width * args.height
    n = trainer.n
    n_tiles = math.ceil(args.width / 16) * math.ceil(args.height / 16)
    m_avg = float(np.mean(pairs)) if pairs else 0.0
    dom_ms = float(np.mean(dom_times)) if dom_times else float(np.mean(singles[dom]))
    dom_bytes = stage_bytes(dom, n, walked, P, n_tiles, n_vis_view, B // world)
    peaks = measured_peaks()
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    traffic, traffic_src = profiled_traffic(dom, args)
    issue, issue_src = profiled_issue(dom, args)
    roofline = {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1),
                "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4),
                "peak_source": peaks["source"], "traffic": traffic,
                "traffic_source": traffic_src,
                "bytes_per_launch": dom_bytes, "avg_launch_ms": round(dom_ms, 4),
                "launches_timed": len(dom_times),
                # the kernel is instruction-issue-bound, not HBM-bound: its
                # issue-slot occupancy from the same capture
                "issue_slots_busy": {"frac": issue, "source": issue_src}}

    # whole-step algorithmic bytes against the same peak
    for st in trainer.last_stats:
        st.walked = walked
    step_bytes = trainer.bytes_per_step([views[0]] * len(trainer.last_stats),
                                        trainer.last_stats)
    step_bytes = max_over_ranks(step_bytes, world)

    # ----------------------------------------------------------------- e2e
    e2e = None
    if not args.no_e2e:
        pinned = [t.pin_memory() for t in targets_u8]

        def e2e_step(i):
            # the step's pinned host images through the public call: the
            # trainer copies them host->device while it projects and bins
            idx = shard(batch_indices(i, B, len(views)), rank, world)
            loss = trainer.train_step([views[j] for j in idx], [pinned[j] for j in idx], B)
            return float(loss.item())                     # device -> host every step

        e2e_step(0)
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            e2e_step(first + args.steps + i)
        trainer.synchronize_params()
        e1.record()
        torch.cuda.synchronize()
        e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
        per_rank_views = B // world
        e2e = {"value": round(1000.0 / e_ms, 3), "unit": "steps/s", "ms_per_step": round(e_ms, 3),
               "h2d_bytes_per_step": per_rank_views * args.width * args.height * 3 * world,
               "d2h_bytes_per_step": 4 * world, "api": "metal_gauss_b200.engine.Trainer.train_step"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.cfg5_shard:
        cpu = cpu_baseline(args, p, views, targets_u8)
    peak_gb = max_over_ranks(torch.cuda.max_memory_allocated(dev) / 1e9, world)

    if rank == 0:
        clk = clocks.summary()
        out = {
            "metric": CFG5_METRIC if args.cfg5_shard else METRIC,
            "value": round(1000.0 / ms, 3), "unit": "steps/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": CFG5_WORKLOAD if args.cfg5_shard else WORKLOAD,
                       "n_gaussians": n, "width": args.width,
                       "height": args.height, "global_batch": B, "views_per_gpu": B // world,
                       "parallelism": f"dp{world}" if world > 1 else "single",
                       "optimizer": "dense Adam" if args.dense_adam else "selective Adam",
                       "l2": "no flush: inputs larger than L2 (parameters + Adam state "
                             f"{3 * 59 * n * 4 / 1e6:.0f} MB, uint8 targets "
                             f"{len(targets) * P * 3 / 1e6:.0f} MB)"},
            "roofline": roofline,
            "step_hbm": {"algorithmic_bytes": step_bytes,
                         "achieved_gbs": round(step_bytes / (ms * 1e-3) / 1e9, 1),
                         "frac": round(step_bytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)},
            "stages_ms": {k: round(float(np.sum(v)) / n_instr, 4) for k, v in stage_ms.items()},
            "pairs_per_view": int(m_avg), "walked_entries_per_view": int(walked),
            "loss": round(loss_val, 6),
            "e2e": e2e, "cpu_baseline": cpu, "gpu_launches": int(launches),
            "clocks": clk, "device_error": int(dev_err),
            "peak_device_memory_gb": round(peak_gb, 2),
        }
        if coll:
            out["collectives_ms"] = coll
        if args.cfg5_shard:
            out["cpu_baseline"] = {"unavailable": "cfg5's CPU baseline is not sampled (the "
                                                  "default cfg3 line carries the CPU baseline)"}
        emit(out)
    if dev_err:
        raise SystemExit(f"device error {dev_err} during the timed steps: "
                         f"{_lib.DEVICE_ERRORS.get(dev_err, 'unknown')}")


def run_render(args, rank, world, local):
    """Forward-only frames/s on cfg4 through renderer.Renderer: each rank
    renders its share of the 256 orbit views (weak in views per rank, no
    collective); one step = every view once. `e2e` adds the device->host copy
    of each frame (rgb + alpha, float32) into pinned memory."""
    from metal_gauss_b200 import _lib, scenes
    from metal_gauss_b200.renderer import Renderer

    dev = torch.device("cuda", local)
    p, views, spec = scenes.config("cfg4", seed=0)
    mine = views[rank::world]
    r = Renderer(p, dev, sh_degree=spec["sh_degree"], antialias=spec["antialias"],
                 background=spec["background"], batch=spec["batch"])
    for _ in range(max(args.warmup, 3)):
        r.render(mine[:spec["batch"]], check=False)
    torch.cuda.synchronize()
    steps = max(1, min(args.steps, 3))
    L = _lib.load()
    barrier(world)
    with ClockSampler(local) as clocks:
        launches0 = L.mg_launch_count()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            # the device error word is checked once after the timed passes
            # (a check per pass synchronises the host between them)
            out = r.render(mine, check=False)
            del out
        e1.record()
        torch.cuda.synchronize()
        launches = (L.mg_launch_count() - launches0) // steps
    _lib.check_device_error("render")
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    W, H = views[0].width, views[0].height
    host = [torch.empty(H, W, 4, dtype=torch.float32).pin_memory() for _ in range(2)]
    barrier(world)
    e0.record()
    for k, (rgb, alpha) in enumerate(r.render(mine, check=False)):
        host[k % 2][..., :3].copy_(rgb, non_blocking=True)
        host[k % 2][..., 3].copy_(alpha, non_blocking=True)
    _lib.check_device_error("render")    # before the frames count as delivered
    e1.record()
    torch.cuda.synchronize()
    e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    if rank == 0:
        frames = len(views)
        emit({
            "metric": "render frames/s (forward only) at 1920x1080, 3M Gaussians, antialias",
            "value": round(1000.0 * frames / ms, 2), "unit": "frames/s", "n_gpus": world,
            "steps": steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 3),
            "ms_per_frame": round(ms / frames, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "cfg4: 3M heavy-tailed Gaussians, SH3, 1920x1080, fov 60, "
                                   "antialias, 256 orbit views per step sharded over the GPUs",
                       "batch_views": spec["batch"],
                       "l2": "no flush: Gaussians (3M x 236 B) larger than L2"},
            "e2e": {"value": round(1000.0 * frames / e_ms, 2), "unit": "frames/s",
                    "h2d_bytes_per_step": 0, "d2h_bytes_per_step": frames * W * H * 16,
                    "api": "metal_gauss_b200.renderer.Renderer.render"},
            "gpu_launches": int(launches), "clocks": clocks.summary(),
        })


# ----------------------------------------------------------- CPU (oracle)

def cpu_view_step(op, params_np, view, target, batch):
    """One view of the training step on the host with the CPU oracle: render,
    loss, backward, activation chain. Returns (loss, grads dict, visible)."""
    means, quats = params_np["means"], params_np["quats"]
    scales = np.exp(params_np["log_scales"]).astype(np.float32)
    opac = (1.0 / (1.0 + np.exp(-params_np["logit_opac"]))).astype(np.float32)
    rgb, alpha, st = op.render(means, quats, scales, opac, params_np["sh_dc"], view.K.numpy(),
                               view.viewmat.numpy(), view.width, view.height, sh_degree=3,
                               sh_rest=params_np["sh_rest"], background=None)
    loss, grad_rgb = op.l1_ssim_loss(rgb, target)
    g = op.render_backward(st, (grad_rgb / batch).astype(np.float32), None)
    grads = {"means": g["means"], "quats": g["quats"], "log_scales": g["scales"] * scales,
             "logit_opac": g["opacities"] * opac * (1 - opac), "sh_dc": g["sh"],
             "sh_rest": g["sh_rest"]}
    return loss / batch, grads, st["pre"]["valid"].astype(bool)


def cpu_adam(op, params_np, grads, visible, state, lrs):
    for name, lr in lrs.items():
        p = params_np[name]
        st = state.setdefault(name, (np.zeros_like(p), np.zeros_like(p),
                                     np.zeros(p.shape[0], np.float32)))
        op.selective_adam_step(p, np.ascontiguousarray(grads[name], np.float32), st[0], st[1],
                               st[2], visible, lr)


def cpu_step(op, params_np, views, targets_u8, idx, batch, state, lrs):
    """One whole training step on the host: every view of the batch `idx`
    rendered, lossed and back-propagated (gradients summed), then one
    selective Adam update on the views' union visibility. Returns
    (seconds in the views, seconds in Adam)."""
    acc, vis = None, None
    t = time.perf_counter()
    for j in idx:
        tgt = targets_u8[j].numpy().astype(np.float32) / np.float32(255.0)
        _, grads, v = cpu_view_step(op, params_np, views[j], tgt, batch)
        if acc is None:
            acc, vis = grads, v.copy()
        else:
            for k in acc:
                acc[k] += grads[k]
            vis |= v
    t_views = time.perf_counter() - t
    t = time.perf_counter()
    cpu_adam(op, params_np, acc, vis.astype(np.uint8), state, lrs)
    return t_views, time.perf_counter() - t


def cpu_baseline(args, p, views, targets_u8, max_views: int = 1) -> dict:
    """The oracle (the reference's algorithm restated in C, OpenMP over all host
    cores) on a bounded sample, to keep the default GPU run short:
    `max_views` view(s) of the step plus the selective Adam update over all 1M
    Gaussians, scaled to steps/s of the whole 8-view step (the reference arm,
    --impl reference, runs whole steps)."""
    import oracle as op
    from metal_gauss_b200.engine import DEFAULT_LRS
    params_np = {k: np.ascontiguousarray(v.numpy(), np.float32) for k, v in p.items()}
    t_views, t_adam = cpu_step(op, params_np, views, targets_u8, list(range(max_views)),
                               args.batch, {}, DEFAULT_LRS)
    t_view = t_views / max_views
    step_s = args.batch * t_view + t_adam
    return {"value": round(1.0 / step_s, 5), "unit": "steps/s", "cores": os.cpu_count(),
            "kind": "port",
            "sample": f"{max_views} of the {args.batch} views of one step (fwd+loss+bwd, "
                      f"{t_view:.2f} s each) + selective Adam over all "
                      f"{args.n_gaussians} Gaussians ({t_adam:.2f} s); steps/s = "
                      f"1 / ({args.batch} x view + Adam)",
            "cpu_model": _cpu_model(), "torch_ref": {"unavailable": TORCH_REF_UNAVAILABLE}}


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args, rank, world):
    """--impl reference: the reference's algorithm (CPU oracle, all host
    threads) on the same workload and metric, rank 0 only. Each timed step is
    the whole step: all `batch` views rendered, lossed and back-propagated,
    then selective Adam on their union visibility. Warm-up steps run one view
    each (they only warm the host's caches and thread pool). Timing stops once
    --cpu-budget-s seconds have gone into timed steps; `steps` reports how
    many ran."""
    if rank != 0:
        return
    import oracle as op
    from metal_gauss_b200.engine import DEFAULT_LRS
    op.build()
    p, views, spec, targets_u8 = workload(args)
    params_np = {k: np.ascontiguousarray(v.numpy(), np.float32) for k, v in p.items()}
    state: dict = {}
    for i in range(args.warmup):
        cpu_step(op, params_np, views, targets_u8, batch_indices(i, args.batch, len(views))[:1],
                 args.batch, state, DEFAULT_LRS)
    times = []
    t_region = time.perf_counter()
    for i in range(args.steps):
        idx = batch_indices(args.warmup + i, args.batch, len(views))
        t_views, t_adam = cpu_step(op, params_np, views, targets_u8, idx, args.batch, state,
                                   DEFAULT_LRS)
        times.append(t_views + t_adam)
        if time.perf_counter() - t_region > args.cpu_budget_s:
            break
    region_s = time.perf_counter() - t_region
    done = len(times)
    step_s = region_s / done
    value = 1.0 / step_s
    emit({
        "impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": "steps/s",
        "n_gpus": world, "steps": done, "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "n_gaussians": args.n_gaussians, "width": args.width,
                   "height": args.height, "global_batch": args.batch, "views_per_gpu": args.batch,
                   "parallelism": "single", "optimizer": "selective Adam"},
        "timed_region_s": round(region_s, 2),
        "cpu_baseline": {"value": round(value, 5), "unit": "steps/s", "cores": os.cpu_count(),
                         "kind": "port",
                         "sample": f"{done} whole steps of {args.batch} views each (fwd+loss+bwd "
                                   "of every view, then selective Adam on their union "
                                   "visibility); warm-up steps one view each; CPU oracle (C, "
                                   "OpenMP, all host threads)",
                         "cpu_model": _cpu_model(),
                         "torch_ref": {"unavailable": TORCH_REF_UNAVAILABLE}},
        "e2e": {"value": round(value, 5), "unit": "steps/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    })


_JSON_FD = None


def emit(obj: dict) -> None:
    """Write the one result line to the process's original stdout (libraries
    such as NCCL print banners to stdout, which is sent to stderr instead)."""
    line = (json.dumps(obj) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(line.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, line)


def main():
    global _JSON_FD
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    args = parse()
    rank, world, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.render:
            run_render(args, rank, world, local)
        else:
            run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

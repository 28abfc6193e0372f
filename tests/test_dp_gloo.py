"""The data-parallel host logic on CPU ranks (gloo, world size 2): each rank
back-propagates its shard of the batch with the CPU oracle into the flat
gradient layout, dp.exchange sums it, and every rank must end with the
single-process sum over the whole batch, including the union visibility.
A rank that dies is detected by its peer through the process-group timeout."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from metal_gauss_b200 import dp, scenes

N, W, H, BATCH = 3000, 64, 48, 4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _run_ranks(fn, extra, world=2, attempts=3):
    """Spawn `world` ranks of fn(rank, world, port, *extra) to completion.
    The port is probed free and then released, so another process can take
    it before rank 0 binds it; a launch that fails is retried on a new port,
    and the last failure is raised."""
    for attempt in range(attempts):
        try:
            mp.start_processes(fn, args=(world, _free_port(), *extra), nprocs=world, join=True,
                               start_method="spawn")
            return
        except (mp.ProcessRaisedException, mp.ProcessExitedException):
            if attempt + 1 == attempts:
                raise


def _scene():
    p, _, _ = scenes.config("cfg3", n=N, seed=5)
    views = scenes.sphere_views(6, 4.0, W, H, 40.0, 2, hemisphere=True)
    g = np.random.default_rng(0)
    targets = [g.random((H, W, 3)).astype(np.float32) for _ in views]
    return {k: v.numpy().astype(np.float32) for k, v in p.items()}, views, targets


def _flat_grad(params, views, targets, idx):
    """Oracle gradient of this rank's views in the trainer's flat layout
    (segments + visibility count tail), and the summed loss."""
    names = ("means", "quats", "log_scales", "logit_opac", "sh_dc", "sh_rest")
    acc = {k: np.zeros_like(params[k]) for k in names}
    vis = np.zeros(N, np.float32)
    loss = 0.0
    scales = np.exp(params["log_scales"]).astype(np.float32)
    opac = (1 / (1 + np.exp(-params["logit_opac"]))).astype(np.float32)
    for j in idx:
        v = views[j]
        rgb, _, st = oracle.render(params["means"], params["quats"], scales, opac,
                                   params["sh_dc"], v.K.numpy(), v.viewmat.numpy(), W, H,
                                   sh_degree=3, sh_rest=params["sh_rest"], background=None)
        l, g_rgb = oracle.l1_ssim_loss(rgb, targets[j])
        g = oracle.render_backward(st, (g_rgb / BATCH).astype(np.float32))
        loss += l / BATCH
        acc["means"] += g["means"]
        acc["quats"] += g["quats"]
        acc["log_scales"] += g["scales"] * scales
        acc["logit_opac"] += g["opacities"] * opac * (1 - opac)
        acc["sh_dc"] += g["sh"]
        acc["sh_rest"] += g["sh_rest"]
        vis += st["pre"]["valid"]
    flat = np.concatenate([acc[k].reshape(-1) for k in names] + [vis])
    return torch.from_numpy(flat), torch.tensor([loss], dtype=torch.float32)


def _worker(rank, world, port, out_dir, step):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    params, views, targets = _scene()
    idx = dp.shard(dp.batch_indices(step, BATCH, len(views)), rank, world)
    flat, loss = _flat_grad(params, views, targets, idx)
    dp.exchange(flat, loss)
    torch.save({"flat": flat, "loss": loss, "idx": idx}, os.path.join(out_dir, f"r{rank}.pt"))
    dist.destroy_process_group()


def test_sharding_covers_the_batch_once():
    idx = dp.batch_indices(3, 8, 100)
    assert idx == list(range(24, 32))
    parts = [dp.shard(idx, r, 4) for r in range(4)]
    assert sum(parts, []) == idx
    with pytest.raises(ValueError):
        dp.shard(idx, 0, 3)


def test_two_gloo_ranks_sum_to_the_single_process_gradient(tmp_path):
    _run_ranks(_worker, (str(tmp_path), 1))
    r0 = torch.load(tmp_path / "r0.pt")
    r1 = torch.load(tmp_path / "r1.pt")
    assert r0["idx"] != r1["idx"]
    assert torch.equal(r0["flat"], r1["flat"]) and torch.equal(r0["loss"], r1["loss"])
    params, views, targets = _scene()
    ref, ref_loss = _flat_grad(params, views, targets, dp.batch_indices(1, BATCH, len(views)))
    rel = float((r0["flat"] - ref).norm() / ref.norm())
    assert rel < 1e-5
    assert abs(float(r0["loss"]) - float(ref_loss)) < 1e-6
    vis = r0["flat"][-N:]
    assert float(vis.max()) <= BATCH and float((vis > 0).sum()) > 0


def _dying_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    flat = torch.ones(16)
    loss = torch.zeros(1)
    dp.exchange(flat, loss)                       # step 1: both ranks
    if rank == 1:
        os._exit(0)                               # rank 1 leaves between steps
    try:
        dp.exchange(flat, loss)                   # step 2: rank 0 alone
        status = "completed"
    except Exception as e:                        # noqa: BLE001
        status = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "status.txt"), "w") as f:
        f.write(status)
    os._exit(0)


def test_a_dead_rank_is_detected_by_its_peer(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_dying_worker, args=(2, port, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(120)
    status = (tmp_path / "status.txt").read_text()
    assert status.startswith("error"), status


def _shard_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    n_pad, width = 8, 3
    g = torch.arange(n_pad * width, dtype=torch.float32) * (rank + 1)   # rank's gradient
    p = torch.ones(n_pad * width)                                     # replicated params
    dp.reduce_scatter_segment(g, None)
    lo, hi = dp.shard_rows(n_pad, rank, world)
    p[lo * width:hi * width] -= 0.5 * g[lo * width:hi * width]        # update own shard only
    dp.all_gather_segment(p, None)
    torch.save(p, os.path.join(out_dir, f"p{rank}.pt"))
    dist.destroy_process_group()


def test_sharded_update_matches_the_replicated_one(tmp_path):
    """ZeRO-1 plumbing: reduce-scatter of a gradient segment, an update on
    each rank's row shard, all-gather of the parameters."""
    _run_ranks(_shard_worker, (str(tmp_path),))
    p0, p1 = torch.load(tmp_path / "p0.pt"), torch.load(tmp_path / "p1.pt")
    ref = 1.0 - 0.5 * (torch.arange(24, dtype=torch.float32) * 3)     # sum over ranks 1 + 2
    assert torch.equal(p0, p1) and torch.allclose(p0, ref)


def _zero_exchange_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    # a flat buffer of two exchange groups of different sizes (the trainer's
    # geometry and SH groups), each a multiple of the world size
    ranges = [(0, 8), (8, 32)]
    x = dp.ZeroExchange(ranges)
    g = torch.arange(32, dtype=torch.float32) * (rank + 1)     # this rank's gradient
    p = torch.ones(32)                                        # replicated parameters
    works = [x.reduce_scatter(g, k) for k in range(2)]        # both groups in flight
    owned = [x.owned(k) for k in range(2)]
    for k in (1, 0):                                          # completed in any order
        works[k].wait()
        a, b = owned[k]
        p[a:b] -= 0.5 * g[a:b]                                # update the rank's chunk only
    gathers = [x.all_gather(p, k) for k in range(2)]
    for w in gathers:
        w.wait()
    torch.save({"p": p, "owned": owned}, os.path.join(out_dir, f"z{rank}.pt"))
    dist.destroy_process_group()


def test_grouped_zero_exchange_matches_the_replicated_update(tmp_path):
    """ZeRO-1 over two exchange groups (dp.ZeroExchange, as the trainer's
    geometry and SH segments): each rank owns chunk r of every group, the
    asynchronous reduce-scatters, chunk updates and all-gathers leave every
    rank with the replicated update."""
    _run_ranks(_zero_exchange_worker, (str(tmp_path),))
    z0, z1 = torch.load(tmp_path / "z0.pt"), torch.load(tmp_path / "z1.pt")
    assert z0["owned"] == [(0, 4), (8, 20)] and z1["owned"] == [(4, 8), (20, 32)]
    ref = 1.0 - 0.5 * (torch.arange(32, dtype=torch.float32) * 3)     # sum over ranks 1 + 2
    assert torch.equal(z0["p"], z1["p"]) and torch.allclose(z0["p"], ref)

"""Data-parallel training on 2 GPUs (NCCL): sharded (ZeRO-1, with the
overlapped per-group exchange) and replicated optimizer steps both equal the
single-GPU steps on the same batches over two consecutive steps (the second
starts while the first's parameter all-gathers are in flight), and the
ranks' parameters stay identical. Needs >= 2 GPUs; skipped otherwise."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

N, W, H, BATCH = 20000, 160, 120, 4


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup():
    from metal_gauss_b200 import scenes
    p, _, _ = scenes.config("cfg3", n=N, seed=3)
    views = scenes.sphere_views(8, 4.0, W, H, 40.0, 4, hemisphere=True)
    g = torch.Generator().manual_seed(0)
    targets = [torch.rand(H, W, 3, generator=g) for _ in views]
    return p, views, targets


def _run(rank, world, port, out, shard):
    from metal_gauss_b200 import dp
    from metal_gauss_b200.engine import SEGMENTS, Trainer
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
    p, views, targets = _setup()
    tr = Trainer(p, f"cuda:{rank}", shard_optimizer=shard)
    tg = [t.cuda(rank) for t in targets]
    idx = dp.shard(dp.batch_indices(0, BATCH, len(views)), rank, world)
    idx2 = dp.shard(dp.batch_indices(1, BATCH, len(views)), rank, world)
    loss = float(tr.train_step([views[j] for j in idx], [tg[j] for j in idx], BATCH))
    # a second step: the first step's parameter all-gathers are still in
    # flight when it starts (the overlapped exchange), and it must see them
    loss2 = float(tr.train_step([views[j] for j in idx2], [tg[j] for j in idx2], BATCH))
    tr.synchronize_params()
    # the gradient elements this rank holds summed: its chunks of the flat
    # parameter region under ZeRO-1 (one per exchange group), everything
    # otherwise
    grads = {}
    for c_lo, c_hi in tr.owned_ranges():
        for k, w in SEGMENTS:
            o = tr.offsets[k]
            b, e = max(c_lo, o) - o, min(c_hi, o + w * tr.n) - o
            if e > b:
                grads.setdefault(k, []).append((b, tr.G[o + b:o + e].cpu()))
    torch.save({"params": {k: v.cpu() for k, v in tr.state_dict().items()}, "loss": loss,
                "loss2": loss2, "grads": grads},
               os.path.join(out, f"{'s' if shard else 'r'}{world}_{rank}.pt"))
    if world > 1:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("shard", [True, False])
def test_two_ranks_match_one(tmp_path, shard):
    mp.start_processes(_run, args=(1, _port(), str(tmp_path), shard), nprocs=1, join=True,
                       start_method="spawn")
    mp.start_processes(_run, args=(2, _port(), str(tmp_path), shard), nprocs=2, join=True,
                       start_method="spawn")
    tag = "s" if shard else "r"
    one = torch.load(tmp_path / f"{tag}1_0.pt")
    ranks = [torch.load(tmp_path / f"{tag}2_{r}.pt") for r in range(2)]
    for k in one["params"]:
        assert torch.equal(ranks[0]["params"][k], ranks[1]["params"][k]), k   # replicas agree
    for k in one["params"]:   # two steps on two ranks equal two steps on one
        rel = float((ranks[0]["params"][k] - one["params"][k]).norm() /
                    one["params"][k].norm().clamp_min(1e-30))
        assert rel < 1e-6, (k, rel)
    for r in ranks:
        assert abs(r["loss"] - one["loss"]) < 1e-5
        assert abs(r["loss2"] - one["loss2"]) < 1e-5
        for k, chunks in r["grads"].items():
            for b, g in chunks:
                ref = one["grads"][k][0][1][b:b + g.numel()]
                rel = float((g - ref).norm() / ref.norm().clamp_min(1e-30))
                assert rel < 1e-5, (k, rel)

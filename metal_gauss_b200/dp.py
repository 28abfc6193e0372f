"""Data-parallel plumbing for the batched trainer: which views a rank renders
and the collectives of a step.

The reference has no distributed code (one view per step on one device,
train.py:352-402). Here a step's batch of views is split into equal
contiguous shards, one per rank, and every rank holds the full Gaussian set.
After its views are back-propagated, the optimizer is sharded (ZeRO-1, the
default with several ranks): the visibility counts and the loss (the tail of
the flat gradient buffer) are all-reduced, the parameter gradient is
reduce-scattered so each rank holds the sum of its own contiguous chunk, each
rank runs Adam on that chunk only, and the updated parameters are
all-gathered in place. `exchange` (one all-reduce of the whole gradient, every
rank then running the full Adam) is the replicated alternative. NCCL over
NVLink on the GPUs; gloo in the CPU tests, which has no reduce-scatter, sums
with an all-reduce instead.
"""

from __future__ import annotations

import torch


def batch_indices(step: int, batch: int, n_views: int) -> list[int]:
    """The global batch of step `step`: `batch` consecutive views, wrapping."""
    return [(step * batch + j) % n_views for j in range(batch)]


def shard(indices: list[int], rank: int, world: int) -> list[int]:
    """This rank's contiguous share of a batch (the batch must divide evenly,
    so every rank renders the same number of views)."""
    if len(indices) % world:
        raise ValueError(f"batch of {len(indices)} views does not split over {world} ranks")
    per = len(indices) // world
    return indices[rank * per:(rank + 1) * per]


def world_size(group=None) -> int:
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group)
    return 1


def exchange(flat_grad: torch.Tensor, loss: torch.Tensor, group=None) -> None:
    """Sum the flat gradient (with its visibility-count tail) and the loss
    over all ranks, in place. Every rank makes exactly these two calls in
    this order every step."""
    if world_size(group) == 1:
        return
    import torch.distributed as dist
    dist.all_reduce(flat_grad, op=dist.ReduceOp.SUM, group=group)
    dist.all_reduce(loss, op=dist.ReduceOp.SUM, group=group)


def rank(group=None) -> int:
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group)
    return 0


def shard_rows(n_pad: int, rank_: int, world: int) -> tuple[int, int]:
    """Row range [lo, hi) of the Gaussians whose optimizer state this rank
    owns; n_pad is a multiple of world."""
    per = n_pad // world
    return rank_ * per, (rank_ + 1) * per


def reduce_scatter_segment(seg: torch.Tensor, group=None) -> None:
    """Sum a (rows x width) segment over ranks, leaving rank r's row shard
    summed in place (other rows are left undefined). NCCL does it as an
    in-place reduce-scatter; gloo (CPU tests), which has none, as an
    all-reduce."""
    import torch.distributed as dist
    world = world_size(group)
    if world == 1:
        return
    if dist.get_backend(group) == "nccl":
        chunk = seg.numel() // world
        r = rank(group)
        dist.reduce_scatter_tensor(seg[r * chunk:(r + 1) * chunk], seg, group=group)
    else:
        dist.all_reduce(seg, group=group)


def all_gather_segment(seg: torch.Tensor, group=None) -> None:
    """Every rank's row shard of a segment, gathered in place on all ranks."""
    import torch.distributed as dist
    world = world_size(group)
    if world == 1:
        return
    chunk = seg.numel() // world
    r = rank(group)
    dist.all_gather_into_tensor(seg, seg[r * chunk:(r + 1) * chunk].clone()
                                if dist.get_backend(group) != "nccl"
                                else seg[r * chunk:(r + 1) * chunk], group=group)


def all_reduce_(t: torch.Tensor, group=None) -> None:
    import torch.distributed as dist
    if world_size(group) > 1:
        dist.all_reduce(t, group=group)

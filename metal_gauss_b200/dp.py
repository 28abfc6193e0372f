"""Data-parallel plumbing for the batched trainer: which views a rank renders
and the one gradient exchange per step.

The reference has no distributed code (one view per step on one device,
train.py:352-402). Here a step's batch of views is split into equal
contiguous shards, one per rank; every rank holds the full Gaussian set; after
its views are back-propagated the flat gradient buffer -- which also carries
each Gaussian's per-rank visibility count -- is summed across ranks in one
all-reduce (NCCL over NVLink on the GPUs, gloo in the CPU tests), together
with the loss.
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

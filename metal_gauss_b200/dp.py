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


class ZeroExchange:
    """The ZeRO-1 exchange of a flat fp32 gradient / parameter pair whose
    segments form `ranges` = [(lo, hi), ...] exchange groups (the trainer's:
    the geometry segments, then the SH segments), each (hi - lo) a multiple of
    the world size. Each group is reduce-scattered, updated and all-gathered
    on a process group of its own, so a small group's collectives never queue
    behind a large group's on one communicator's stream, and every call is
    asynchronous: it returns a work handle whose `wait()` makes the current
    CUDA stream (nothing on the host) wait for it. Rank r owns chunk r of
    every group. Every rank must build it, and call its methods, in the same
    order."""

    def __init__(self, ranges, group=None):
        import torch.distributed as dist
        self.world, self.rank = world_size(group), rank(group)
        for lo, hi in ranges:
            if (hi - lo) % self.world:
                raise ValueError(f"exchange group [{lo}, {hi}) does not split over "
                                 f"{self.world} ranks")
        self.ranges = list(ranges)
        self.backend = dist.get_backend(group)
        ranks = list(range(self.world)) if group is None else dist.get_process_group_ranks(group)
        # one communicator per exchange group (new_group is collective)
        self.groups = [dist.new_group(ranks, backend=self.backend) for _ in self.ranges]

    def owned(self, k: int) -> tuple[int, int]:
        """Flat [lo, hi) of exchange group k that this rank updates."""
        lo, hi = self.ranges[k]
        chunk = (hi - lo) // self.world
        return lo + self.rank * chunk, lo + (self.rank + 1) * chunk

    def reduce_scatter(self, flat: torch.Tensor, k: int):
        """Sum group k of `flat` over ranks, leaving this rank's chunk summed
        in place (the rest of the group is left undefined). gloo, which has no
        reduce-scatter, sums the whole group with an all-reduce."""
        import torch.distributed as dist
        lo, hi = self.ranges[k]
        seg = flat[lo:hi]
        if self.backend == "nccl":
            a, b = self.owned(k)
            return dist.reduce_scatter_tensor(flat[a:b], seg, group=self.groups[k],
                                              async_op=True)
        return dist.all_reduce(seg, group=self.groups[k], async_op=True)

    def all_gather(self, flat: torch.Tensor, k: int):
        """Every rank's chunk of group k of `flat`, gathered in place."""
        import torch.distributed as dist
        lo, hi = self.ranges[k]
        a, b = self.owned(k)
        src = flat[a:b] if self.backend == "nccl" else flat[a:b].clone()
        return dist.all_gather_into_tensor(flat[lo:hi], src, group=self.groups[k],
                                           async_op=True)

    def all_reduce(self, t: torch.Tensor, k: int = 0):
        import torch.distributed as dist
        return dist.all_reduce(t, group=self.groups[k], async_op=True)

"""Multi-GPU sharding of the hot path: one process per GPU, the batch (MLP
rows, image row bands) split into contiguous ranges, each rank computing its
range with no cross-rank traffic, and one all-gather of the results at the
end (NCCL over NVLink on GPUs; gloo in the CPU tests).

The reference has no multi-device execution at all; this is the B200
scale-out of its data-parallel operators. Nothing here touches device
memory of another GPU: each rank's kernels read only local tensors, and the
exchange is a library collective.
"""
from __future__ import annotations

import torch


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of `rank`'s contiguous share of n units: the first
    n % world ranks get one unit more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a world of {world}")
    if n < 0:
        raise ValueError("n must be >= 0")
    base, extra = divmod(n, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def shard_sizes(n: int, world: int) -> list[int]:
    return [shard_range(n, world, r)[1] - shard_range(n, world, r)[0] for r in range(world)]


def all_gather_rows(local: torch.Tensor, n: int, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Concatenates every rank's `local` block (rank order, leading dimension
    = its shard of n rows) into an [n, ...] tensor on every rank, with one
    all_gather_into_tensor. Unequal shards are padded to the largest and
    trimmed."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    sizes = shard_sizes(n, world)
    if local.shape[0] != sizes[rank]:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, its shard of {n} is {sizes[rank]}")
    tail = tuple(local.shape[1:])
    m = max(sizes) if sizes else 0
    if all(s == m for s in sizes):
        if out is None:
            out = torch.empty((n,) + tail, dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
        return out
    padded = torch.zeros((m,) + tail, dtype=local.dtype, device=local.device)
    padded[:local.shape[0]] = local
    full = torch.empty((m * world,) + tail, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(full, padded, group=group)
    if out is None:
        out = torch.empty((n,) + tail, dtype=local.dtype, device=local.device)
    for r, s in enumerate(sizes):
        b, _ = shard_range(n, world, r)
        out[b:b + s] = full[r * m:r * m + s]
    return out


def sharded_map(m, x: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Evaluates Map `m` on this rank's rows of x ([n, IN], the full batch or
    any tensor indexable by row) and all-gathers [n, OUT] on every rank."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n = x.shape[0]
    b, e = shard_range(n, world, rank)
    local = m(x[b:e])
    local = local.as_tensor("torch") if hasattr(local, "as_tensor") else local
    return all_gather_rows(local, n, group=group, out=out)


def sharded_render(renderer, pose9, width: int, height: int, group=None, **kw) -> torch.Tensor:
    """Renders this rank's band of image rows with a VolumeRenderer and
    all-gathers the [height, width, 4] RGBA image on every rank."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    b, e = shard_range(height, world, rank)
    band = renderer.render(pose9, width, height, row_begin=b, row_end=e, **kw)
    return all_gather_rows(band, height, group=group)

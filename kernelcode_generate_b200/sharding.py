"""Partitioning of the three kernels across the GPUs of one node, and the optional output gather.

The work splits with no exchange: matmul by contiguous row blocks of M, attention by (b, h) pairs,
conv2d by batch. Every rank computes its block from its own inputs; when a caller wants the whole
result as one tensor, `gather_rows` all-gathers the blocks (NCCL over NVLink on GPUs, gloo on the
host) along the partitioned dimension.
"""

from __future__ import annotations


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [begin, end) of `total` owned by `rank`; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    return total * rank // world, total * (rank + 1) // world


def gather_rows(local, total: int, group=None):
    """All-gather row blocks split by `shard_range(total, rank, world)` along dim 0.

    `local` holds this rank's rows (dim 0 = end - begin, any trailing shape, same on all ranks).
    Returns the full tensor (dim 0 = total) on every rank. Blocks are padded to the largest block
    so the collective moves equal-size pieces (NCCL `all_gather_into_tensor`; a list all-gather on
    backends without it), then the padding is dropped.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    begin, end = shard_range(total, rank, world)
    if local.shape[0] != end - begin:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, its block is {end - begin}")
    if world == 1:
        return local
    block = -(-total // world)  # the largest block
    padded = local.new_zeros((block,) + tuple(local.shape[1:]))
    padded[: end - begin].copy_(local)
    if dist.get_backend(group) == "nccl":
        out = local.new_empty((world * block,) + tuple(local.shape[1:]))
        dist.all_gather_into_tensor(out, padded.contiguous(), group=group)
        pieces = list(out.split(block, dim=0))
    else:
        pieces = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(pieces, padded.contiguous(), group=group)
    parts = []
    for r in range(world):
        b, e = shard_range(total, r, world)
        parts.append(pieces[r][: e - b])
    return torch.cat(parts, dim=0)

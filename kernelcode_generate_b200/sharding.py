"""Partitioning of the three kernels across the GPUs of one node, and the optional output gather.

The work splits with no exchange: matmul by contiguous row blocks of M, attention by (b, h) pairs,
conv2d by batch. Every rank computes its block from its own inputs; when a caller wants the whole
result as one tensor, `gather_rows` all-gathers the blocks (NCCL over NVLink on GPUs, gloo on the
host) along the partitioned dimension.

`matmul_rows_from_host` is the multi-GPU form of the reference's host-buffer call
(kernel/matmul/inputs_dynamic_tile_dynamic.py:233-251 runs the compiled kernel on host arrays):
every rank needs all of B, but B crosses the host link only once for the whole job. Each rank
uploads 1/N of B's rows, one NCCL all-gather over NVLink replicates B on every GPU, and the
reference-facing slot entry then runs the rank's row block from host memory (upload of its A
rows, kernel, download of its C rows, pipelined in row blocks inside the entry).
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
    if end - begin == block:
        padded = local
    else:
        padded = local.new_zeros((block,) + tuple(local.shape[1:]))
        padded[: end - begin].copy_(local)
    if dist.get_backend(group) == "nccl":
        out = local.new_empty((world * block,) + tuple(local.shape[1:]))
        dist.all_gather_into_tensor(out, padded.contiguous(), group=group)
        pieces = list(out.split(block, dim=0))
    else:
        pieces = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(pieces, padded.contiguous(), group=group)
    if total % world == 0 and dist.get_backend(group) == "nccl":
        return out  # equal blocks: no padding to drop
    parts = []
    for r in range(world):
        b, e = shard_range(total, r, world)
        parts.append(pieces[r][: e - b])
    return torch.cat(parts, dim=0)


_REPLICA_BUFFERS: dict = {}


def replicate_from_host_shards(host, device, group=None):
    """Whole copy of the host matrix `host` ([R, ...], a torch CPU tensor, pinned for an
    asynchronous upload) on `device` of every rank, with each rank uploading only its rows
    shard_range(R, rank, world) and one all-gather (`gather_rows`: NCCL over NVLink on GPUs)
    filling in the rest. The upload buffer is kept per (device, shape, dtype) and reused; runs on
    the current stream."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    rows = host.shape[0]
    b0, b1 = shard_range(rows, rank, world)
    key = (str(device), tuple(host.shape), host.dtype, world, rank)
    local = _REPLICA_BUFFERS.get(key)
    if local is None:
        local = _REPLICA_BUFFERS[key] = torch.empty((b1 - b0,) + tuple(host.shape[1:]), dtype=host.dtype, device=device)
    local.copy_(host[b0:b1], non_blocking=True)
    if world == 1:
        return local
    return gather_rows(local, rows, group)


def matmul_rows_from_host(out, lhs, rhs, bias, tile_h, tile_w, tile_k, group=None):
    """This rank's share of out = lhs @ rhs (+ bias) from host buffers, B uploaded once per job.

    `out` [rows, N] f32 and `lhs` [rows, K] hold this rank's contiguous row block in host memory
    (torch CPU tensors, pinned for overlapped copies); `rhs` [K, N] is the whole host matrix, of
    which this rank uploads only rows shard_range(K, rank, world); `bias` [N] f32 (host) or None;
    the tile arguments are the reference wrapper's. B is replicated over NVLink
    (`replicate_from_host_shards`), then the reference-facing slot entry runs with lhs and out in
    host memory (its pipelined upload / kernel / download of row blocks) and B in device memory.
    Returns the slot entry's ExecuteResult."""
    import torch

    from . import kernels

    device = torch.device("cuda", torch.cuda.current_device())
    rhs_dev = replicate_from_host_shards(rhs, device, group)
    torch.cuda.current_stream().synchronize()  # the slot entry runs on its own streams
    return kernels.matmul_inputs_dynamic_tile_dynamic_kernel(out, lhs, rhs_dev, bias, tile_h, tile_w, tile_k)

"""Multi-process host logic of the sharded bench path, on CPU with the gloo backend
(world size 2): the shards tile the work exactly, per-rank oracle results assemble into the
single-process result (the partition needs no exchange), and the timing reductions take the
max / sum over ranks."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import bench
import oracle


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("total,world", [(8192, 1), (8192, 2), (8192, 8), (128, 8), (7, 3), (5, 8)])
def test_shard_ranges_tile_the_work(total, world):
    ranges = [bench.shard_range(total, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == total
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0 and a0 <= a1
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1


def _worker(rank, world, port, results):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(3)
        a = rng.standard_normal((37, 24), dtype=np.float32)
        b = rng.standard_normal((24, 19), dtype=np.float32)
        r0, r1 = bench.shard_range(a.shape[0], rank, world)
        part = oracle.matmul(np.ascontiguousarray(a[r0:r1]), b, tiles=(8, 8, 8))
        q, k, v = (rng.standard_normal((2, 3, 40, 16), dtype=np.float32) for _ in range(3))
        b0, b1 = bench.shard_range(6, rank, world)
        shard = lambda x: np.ascontiguousarray(x.reshape(6, 40, 16)[b0:b1]).reshape(1, b1 - b0, 40, 16)  # noqa: E731
        fa = oracle.flash_attention(shard(q), shard(k), shard(v), tiles=(16, 16), scale=0.25, causal=True)
        # assemble on every rank with a gather of variable-size pieces (padded)
        pieces = [None] * world
        dist.all_gather_object(pieces, (r0, part, b0, fa))
        slowest = bench.reduce_max(float(rank + 1), world)
        total = bench.reduce_sum(float(r1 - r0), world)
        if rank == 0:
            results.put((pieces, slowest, total))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_row_and_head_sharding_need_no_exchange():
    world = 2
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    pieces, slowest, total = results.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(3)
    a = rng.standard_normal((37, 24), dtype=np.float32)
    b = rng.standard_normal((24, 19), dtype=np.float32)
    full = oracle.matmul(a, b, tiles=(8, 8, 8))
    assembled = np.concatenate([p[1] for p in sorted(pieces, key=lambda x: x[0])], axis=0)
    np.testing.assert_array_equal(assembled, full)
    q, k, v = (rng.standard_normal((2, 3, 40, 16), dtype=np.float32) for _ in range(3))
    fa_full = oracle.flash_attention(q, k, v, tiles=(16, 16), scale=0.25, causal=True).reshape(6, 40, 16)
    fa_assembled = np.concatenate([p[3].reshape(-1, 40, 16) for p in sorted(pieces, key=lambda x: x[2])], axis=0)
    np.testing.assert_array_equal(fa_assembled, fa_full)
    assert slowest == 2.0 and total == 37.0


def _gather_worker(rank, world, port, results):
    import torch
    import torch.distributed as dist

    from kernelcode_generate_b200.sharding import gather_rows, shard_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        a = rng.standard_normal((37, 24), dtype=np.float32)
        b = rng.standard_normal((24, 19), dtype=np.float32)
        r0, r1 = shard_range(a.shape[0], rank, world)
        part = torch.from_numpy(oracle.matmul(np.ascontiguousarray(a[r0:r1]), b, tiles=(8, 8, 8)))
        mm = gather_rows(part, a.shape[0])
        q, k, v = (rng.standard_normal((2, 3, 40, 16), dtype=np.float32) for _ in range(3))
        b0, b1 = shard_range(6, rank, world)
        shard = lambda x: np.ascontiguousarray(x.reshape(6, 40, 16)[b0:b1]).reshape(1, b1 - b0, 40, 16)  # noqa: E731
        fa = torch.from_numpy(oracle.flash_attention(shard(q), shard(k), shard(v), tiles=(16, 16), scale=0.25, causal=True))
        att = gather_rows(fa.reshape(-1, 40, 16), 6)
        bad = None
        try:
            gather_rows(part[:0] if r1 > r0 else part, a.shape[0])
        except ValueError as exc:
            bad = str(exc)
        if rank == 0:
            results.put((mm.numpy(), att.numpy(), bad))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gather_rows_assembles_the_single_process_result(world):
    """The optional output all-gather: uneven row blocks (37 rows over 2 or 3 ranks, 6 heads over
    3) come back as the single-process result on every rank, bit for bit."""
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    mm, att, bad = results.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(11)
    a = rng.standard_normal((37, 24), dtype=np.float32)
    b = rng.standard_normal((24, 19), dtype=np.float32)
    np.testing.assert_array_equal(mm, oracle.matmul(a, b, tiles=(8, 8, 8)))
    q, k, v = (rng.standard_normal((2, 3, 40, 16), dtype=np.float32) for _ in range(3))
    np.testing.assert_array_equal(att, oracle.flash_attention(q, k, v, tiles=(16, 16), scale=0.25, causal=True).reshape(6, 40, 16))
    assert bad is not None and "block" in bad


def _replicate_worker(rank, world, port, results):
    import torch
    import torch.distributed as dist

    from kernelcode_generate_b200.sharding import replicate_from_host_shards, shard_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(21)
        b = torch.from_numpy(rng.standard_normal((37, 19), dtype=np.float32))
        # Each rank holds only its own rows of B; the rest of its host copy is garbage that must
        # never reach the replica.
        k0, k1 = shard_range(37, rank, world)
        host = torch.full_like(b, float("nan"))
        host[k0:k1] = b[k0:k1]
        first = replicate_from_host_shards(host, torch.device("cpu")).clone()
        second = replicate_from_host_shards(host * 2, torch.device("cpu")).clone()  # buffers reused
        results.put((rank, first.numpy(), second.numpy()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_b_is_replicated_from_one_upload_per_row_block(world):
    """The multi-GPU host-buffer matmul uploads each row of B from one rank only and all-gathers
    it: every rank ends with the whole B, bit for bit, from host copies that hold only its own
    rows (37 rows: uneven blocks over 2 and 3 ranks), and a second call reuses the buffers."""
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_replicate_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = [results.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    b = np.random.default_rng(21).standard_normal((37, 19), dtype=np.float32)
    for _, first, second in got:
        np.testing.assert_array_equal(first, b)
        np.testing.assert_array_equal(second, 2 * b)

"""Data-parallel host logic on CPU: two gloo ranks average their packed dweights.

Mirrors the reference's multi-process CPU tests (tests/test_ddp.py: spawn context, gloo,
free-port rendezvous on 127.0.0.1). Each rank fills a DWeightBucket with rank-specific
values; after all_reduce every rank must hold the same average, bit for bit, and the
averaging must equal what DDP would produce (sum / world).
"""

from __future__ import annotations

import datetime
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from picotron_b200.dist import DWeightBucket


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, results) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        sizes = [4096, 4096, 128, 7]
        bucket = DWeightBucket(sizes, "cpu")
        g = torch.Generator().manual_seed(100 + rank)
        for i, size in enumerate(sizes):
            bucket.slot(i).copy_(torch.randn(size, generator=g))
        bucket.all_reduce()
        results[rank] = [bucket.slot(i).clone() for i in range(len(sizes))]
    finally:
        dist.destroy_process_group()


def test_dweight_bucket_average_over_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        got = {r: results[r] for r in range(world)}
    sizes = [4096, 4096, 128, 7]
    expected = []
    for i, size in enumerate(sizes):
        acc = torch.zeros(size)
        for r in range(world):
            g = torch.Generator().manual_seed(100 + r)
            vals = [torch.randn(s, generator=g) for s in sizes]
            acc += vals[i]
        expected.append(acc / world)
    for i in range(len(sizes)):
        assert torch.equal(got[0][i], got[1][i])  # identical on every rank
        torch.testing.assert_close(got[0][i], expected[i], rtol=1e-6, atol=1e-6)


def test_bucket_slots_are_aligned_views():
    bucket = DWeightBucket([5, 3, 8], "cpu")
    assert bucket.offsets == [0, 8, 12, 20]
    bucket.slot(1).fill_(2.0)
    assert bucket.buffer[8:11].eq(2.0).all() and bucket.buffer[11] == 0
    for i in range(3):
        assert bucket.slot(i).data_ptr() % 16 == 0
    bucket.all_reduce()  # no process group: a no-op


def _async_worker(rank: int, world: int, port: int, results) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        sizes = [64, 64, 5, 64, 64, 64]
        bucket = DWeightBucket(sizes, "cpu")
        g = torch.Generator().manual_seed(200 + rank)
        for i, size in enumerate(sizes):
            bucket.slot(i).copy_(torch.randn(size, generator=g))
        # Buckets in the order a backward produces them (last layers first).
        pending = [bucket.all_reduce_async(4, 6), bucket.all_reduce_async(1, 4),
                   bucket.all_reduce_async(0, 1, average=False)]
        for p in pending:
            p.wait()
        results[rank] = [bucket.slot(i).clone() for i in range(len(sizes))]
    finally:
        dist.destroy_process_group()


def test_async_slot_ranges_over_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_async_worker, args=(r, world, port, results))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
        got = {r: results[r] for r in range(world)}
    sizes = [64, 64, 5, 64, 64, 64]
    per_rank = []
    for r in range(world):
        g = torch.Generator().manual_seed(200 + r)
        per_rank.append([torch.randn(s, generator=g) for s in sizes])
    for i in range(len(sizes)):
        total = per_rank[0][i] + per_rank[1][i]
        expected = total if i == 0 else total / world  # slot 0 was summed, not averaged
        assert torch.equal(got[0][i], got[1][i])
        torch.testing.assert_close(got[0][i], expected, rtol=1e-6, atol=1e-6)


def test_async_rejects_bad_ranges_and_is_a_no_op_without_a_group():
    bucket = DWeightBucket([5, 3], "cpu")
    bucket.slot(0).fill_(1.0)
    bucket.all_reduce_async(0, 2).wait()
    assert bucket.slot(0).eq(1.0).all()
    for first, stop in [(1, 1), (-1, 1), (0, 3)]:
        try:
            bucket.all_reduce_async(first, stop)
        except ValueError:
            continue
        raise AssertionError(f"range [{first}, {stop}) was accepted")

"""Failure detection of the data-parallel dweight exchange, on gloo ranks on CPU.

The reference's data-parallel wrapper relies on the process group's timeout to turn a
missing peer into an error (src/picotron/parallel/ddp.py:56-63, init_process_group with a
timeout). These tests make the failures on the host, with no GPU involved:

* a rank that skips one bucket's all-reduce: the other rank's ``wait`` must raise once the
  short process-group timeout has passed, not hang;
* a rank that exits without taking part: the waiting rank must raise as well;
* a rendezvous that one rank never joins: ``init_process_group`` must raise.

Each scenario runs in spawned child processes with a hard join limit, so a regression shows
up as a failed assertion, never as a hung test run.
"""

from __future__ import annotations

import datetime
import os
import socket
import time

import torch.distributed as dist
import torch.multiprocessing as mp

from picotron_b200.dist import DWeightBucket

PG_TIMEOUT_S = 3.0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _skip_worker(rank: int, port: int, mode: str, results, done) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
    bucket = DWeightBucket([64, 64, 64], "cpu")
    bucket.slot(0).fill_(float(rank + 1))
    # Both ranks agree on the first bucket.
    bucket.all_reduce_async(2, 3).wait()
    if rank == 0:
        t0 = time.monotonic()
        try:
            bucket.all_reduce_async(0, 2).wait()
            results[rank] = ("no error", time.monotonic() - t0)
        except Exception as exc:  # the expected outcome
            results[rank] = (type(exc).__name__ + ": " + str(exc)[:200], time.monotonic() - t0)
        done.set()
    else:
        # Rank 1 never issues the second all-reduce.
        if mode == "stall":
            done.wait(60)  # alive but silent until rank 0 has given up
        results[rank] = ("skipped", 0.0)
    # A group whose collective failed is not torn down collectively; the process just ends.
    os._exit(0)


def _run_skip(mode: str):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        done = manager.Event()
        port = _free_port()
        procs = [ctx.Process(target=_skip_worker, args=(r, port, mode, results, done))
                 for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=90)
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        return dict(results)


def test_skipped_all_reduce_raises_after_the_group_timeout():
    results = _run_skip("stall")
    message, waited = results[0]
    assert message != "no error", "rank 0 completed an all-reduce that rank 1 never issued"
    # It gave up because of the timeout (not at once, and not much later).
    assert PG_TIMEOUT_S * 0.5 <= waited <= PG_TIMEOUT_S + 20, (message, waited)
    assert results[1][0] == "skipped"


def test_all_reduce_with_an_exited_peer_raises():
    results = _run_skip("exit")
    message, waited = results[0]
    assert message != "no error"
    assert waited <= PG_TIMEOUT_S + 20, (message, waited)


def _lonely_rank(port: int, results) -> None:
    t0 = time.monotonic()
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0,
                                world_size=2, timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
        results["outcome"] = ("joined", time.monotonic() - t0)
    except Exception as exc:  # the expected outcome
        results["outcome"] = (type(exc).__name__ + ": " + str(exc)[:200], time.monotonic() - t0)
    os._exit(0)


def test_rendezvous_without_the_second_rank_raises():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        p = ctx.Process(target=_lonely_rank, args=(_free_port(), results))
        p.start()
        p.join(timeout=90)
        if p.is_alive():
            p.kill()
            p.join()
            raise AssertionError("init_process_group waited for ever for the missing rank")
        assert p.exitcode == 0
        message, waited = results["outcome"]
    assert message != "joined"
    assert waited <= PG_TIMEOUT_S + 30, (message, waited)

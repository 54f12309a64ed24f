"""Fault-tolerant dispatch on CPU (the multi-GPU failure plan with host-side faults only): a
worker that raises, a worker that stops beating, a rank process that exits mid-item and a rank
that hangs. Every item must be delivered exactly once with the right result."""
import datetime
import multiprocessing as mp
import os
import time

import pytest
import torch.distributed as dist

from qwen3tts.dispatch import StoreQueue, ThreadDispatcher, WorkerFailed


def test_thread_dispatcher_requeues_failed_and_stalled_workers():
    calls = {1: 0, 2: 0}

    def ok(item, beat):
        time.sleep(0.02)
        return item * item

    def raises(item, beat):
        calls[1] += 1
        raise RuntimeError("device lost")

    def stalls(item, beat):
        calls[2] += 1
        time.sleep(0.6)  # no heartbeat for longer than the timeout
        return item * item

    d = ThreadDispatcher([ok, raises, stalls], timeout=0.2, poll=0.01)
    items = list(range(24))
    assert d.run(items) == [i * i for i in items]
    assert set(d.failed) == {1, 2}
    assert "device lost" in d.failed[1] and "heartbeat" in d.failed[2]
    assert calls == {1: 1, 2: 1}
    assert sorted(d.ran) == items


def test_thread_dispatcher_long_item_with_beats_is_kept():
    def slow(item, beat):
        for _ in range(6):
            time.sleep(0.05)
            beat()
        return -item

    d = ThreadDispatcher([slow], timeout=0.15, poll=0.01)
    assert d.run([1, 2]) == [-1, -2] and not d.failed


def test_thread_dispatcher_all_failed():
    def bad(item, beat):
        raise ValueError("no")

    with pytest.raises(WorkerFailed):
        ThreadDispatcher([bad, bad], timeout=1.0, poll=0.01).run([1, 2, 3])


def _rank(port: int, rank: int, world: int, n: int):
    store = dist.TCPStore("127.0.0.1", port, None, False,
                          timeout=datetime.timedelta(seconds=30))
    q = StoreQueue(store, rank, world, n, prefix="t", timeout=0.5, beat=0.05, publish=True,
                   stall_after=0.3)
    first = [True]

    def fn(i):
        if first[0]:
            first[0] = False
            if rank == 2:
                os._exit(3)        # dies holding its first item
            if rank == 1:
                time.sleep(2.5)    # hangs on its first item, no progress reported
        time.sleep(0.02)
        return {"item": i, "square": i * i, "rank": rank}

    out = q.run(fn, poll=0.02)
    store.set(f"out/{rank}", ",".join(str(i) for i in sorted(out)))
    os._exit(0)


def test_store_queue_survives_a_dead_and_a_hung_rank():
    world, n = 3, 30
    server = dist.TCPStore("127.0.0.1", 0, None, True,
                           timeout=datetime.timedelta(seconds=30), wait_for_workers=False)
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank, args=(server.port, r, world, n)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
        assert not p.is_alive()
    assert procs[2].exitcode == 3 and procs[0].exitcode == 0 and procs[1].exitcode == 0
    q = StoreQueue(server, 0, world, n, prefix="t")
    got = q.gather()
    assert [g["square"] for g in got] == [i * i for i in range(n)]
    taken = {}
    for r in (0, 1):
        s = server.get(f"out/{r}").decode()
        for i in (s.split(",") if s else []):
            assert int(i) not in taken  # exactly once
            taken[int(i)] = r
    assert sorted(taken) == list(range(n))
    assert all(got[i]["rank"] == taken[i] for i in range(n))
    assert all(got[i]["rank"] != 2 for i in range(n))

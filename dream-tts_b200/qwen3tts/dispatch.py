"""Fault-tolerant dispatch of independent work items (talker groups, codec chunks) over GPUs.

Items never exchange data (lanes never read each other's cache, crates/qwen3tts/src/
talker.rs:83-84; codec chunks carry their own left context, codec.rs:562-604), so a worker
that fails or stops answering loses nothing that cannot be redone: its unfinished items go back
on the queue and another worker runs them. Every item's result is taken once (the first
completion wins; a late duplicate from a worker that was given up on is dropped). Detection is
on the host: a worker's exception, or no heartbeat for `timeout` seconds; device-side waits
stay bounded inside the kernels themselves.

Two forms:
  * `ThreadDispatcher`: one worker thread per GPU in one process (the reference's engine
    drives its device from one dispatcher thread, crates/tts-nn/src/lib.rs:76-88);
  * `StoreQueue`: one process per GPU (torchrun), items claimed through a shared
    torch.distributed Store (an atomic counter), heartbeats as store counters, ownership moved
    with compare-and-set, results optionally published in the store for rank 0 to gather.
"""
from __future__ import annotations

import collections
import pickle
import threading
import time
from typing import Callable, Optional


class WorkerFailed(RuntimeError):
    pass


class ThreadDispatcher:
    """run(items) -> results in item order. `workers[w](item, beat)` runs one item on worker w's
    device; it may call `beat()` during long work to refresh its heartbeat."""

    def __init__(self, workers: list[Callable], timeout: float = 30.0, poll: float = 0.02):
        if not workers:
            raise ValueError("no workers")
        self.workers, self.timeout, self.poll = workers, timeout, poll
        self.failed: dict[int, str] = {}   # worker -> why it was given up on
        self.ran: dict[int, int] = {}      # item -> worker whose result was taken
        self.attempts: collections.Counter = collections.Counter()

    def run(self, items: list) -> list:
        n = len(items)
        lock = threading.Lock()
        queue = collections.deque(range(n))
        results: list = [None] * n
        have = [False] * n
        current: list[Optional[int]] = [None] * len(self.workers)
        beat_at = [time.monotonic()] * len(self.workers)
        alive = [True] * len(self.workers)

        def requeue(w):
            i = current[w]
            current[w] = None
            if i is not None and not have[i]:
                queue.appendleft(i)

        def body(w):
            def beat():
                with lock:
                    beat_at[w] = time.monotonic()
            while True:
                with lock:
                    while queue and have[queue[0]]:
                        queue.popleft()  # a late duplicate already delivered it
                    if not alive[w] or not queue:
                        return
                    i = queue.popleft()
                    current[w] = i
                    beat_at[w] = time.monotonic()
                    self.attempts[i] += 1
                try:
                    r = self.workers[w](items[i], beat)
                except BaseException as e:  # noqa: BLE001 - any failure retires the worker
                    with lock:
                        if alive[w]:
                            alive[w] = False
                            self.failed[w] = f"raised {type(e).__name__}: {e}"
                            requeue(w)
                    return
                with lock:
                    if not have[i]:
                        results[i], have[i] = r, True
                        self.ran[i] = w
                    if current[w] == i:
                        current[w] = None

        threads = [threading.Thread(target=body, args=(w,), daemon=True)
                   for w in range(len(self.workers))]
        for t in threads:
            t.start()
        while True:
            with lock:
                if all(have):
                    break
                now = time.monotonic()
                for w in range(len(self.workers)):
                    if alive[w] and current[w] is not None and now - beat_at[w] > self.timeout:
                        alive[w] = False
                        self.failed[w] = f"no heartbeat for {self.timeout:.3g} s"
                        requeue(w)
                idle = [w for w in range(len(self.workers))
                        if alive[w] and not threads[w].is_alive()]
                for w in idle:  # finished its loop while items came back: restart it
                    threads[w] = threading.Thread(target=body, args=(w,), daemon=True)
                    threads[w].start()
                if not any(alive):
                    raise WorkerFailed(f"every worker failed: {self.failed}")
            time.sleep(self.poll)
        return results


class StoreQueue:
    """Items 0..n-1 shared by `world` processes through `store` (all ranks construct it with
    the same prefix and n). run(fn) runs items on this rank until every item is done anywhere,
    taking over items whose owner stopped beating for `timeout` seconds; returns this rank's
    results {item: result}. With `publish`, results go into the store for `gather`."""

    def __init__(self, store, rank: int, world: int, n: int, prefix: str = "queue",
                 timeout: float = 30.0, beat: float = 0.2, publish: bool = False,
                 stall_after: Optional[float] = None):
        self.s, self.rank, self.world, self.n = store, rank, world, n
        self.p, self.timeout, self.beat_every, self.publish = prefix, timeout, beat, publish
        # with stall_after, the heartbeat stops while an item has made no progress (no new item
        # and no progress() call) for that long: a hung rank then looks like a dead one
        self.stall_after = stall_after
        self._last_progress = time.monotonic()
        self._stop = threading.Event()
        self._seen: dict[int, tuple[int, float]] = {}  # rank -> (beat count, first seen at)
        self._orphan: dict[int, float] = {}            # item -> first seen without an owner

    def progress(self) -> None:
        """Called by a long-running item to keep this rank's heartbeat going."""
        self._last_progress = time.monotonic()

    def _k(self, *parts) -> str:
        return "/".join([self.p] + [str(x) for x in parts])

    def _beat_loop(self):
        while not self._stop.is_set():
            if self.stall_after is None or time.monotonic() - self._last_progress < self.stall_after:
                self.s.add(self._k("hb", self.rank), 1)
            self._stop.wait(self.beat_every)

    def _stale(self, r: int) -> bool:
        """No heartbeat increment from rank r for `timeout` seconds of this rank's clock."""
        v = self.s.add(self._k("hb", r), 0)
        now = time.monotonic()
        last = self._seen.get(r)
        if last is None or last[0] != v:
            self._seen[r] = (v, now)
            return False
        return now - last[1] > self.timeout

    def _done(self, i: int) -> bool:
        return self.s.check([self._k("done", i)])

    def _claim(self, i: int, expected: str) -> bool:
        me = str(self.rank)
        return self.s.compare_set(self._k("owner", i), expected, me) == me.encode()

    def _run_one(self, fn, i: int, out: dict):
        self._last_progress = time.monotonic()
        r = fn(i)
        # first completion wins: a late duplicate is dropped
        if self.s.compare_set(self._k("done", i), "", str(self.rank)) == str(self.rank).encode():
            out[i] = r
            if self.publish:
                self.s.set(self._k("res", i), pickle.dumps(r))

    def run(self, fn: Callable[[int], object], poll: float = 0.05) -> dict:
        out: dict = {}
        t = threading.Thread(target=self._beat_loop, daemon=True)
        self.s.add(self._k("hb", self.rank), 1)
        t.start()
        try:
            while True:
                i = self.s.add(self._k("next"), 1) - 1
                if i >= self.n:
                    break
                if self._claim(i, ""):  # lost only to a rank that took it over as an orphan
                    self._run_one(fn, i, out)
            # recovery: items claimed by ranks that stopped beating
            while True:
                pending = [i for i in range(self.n) if not self._done(i)]
                if not pending:
                    break
                for i in pending:
                    if not self.s.check([self._k("owner", i)]):
                        # counted out but never owned: its claimer died in between, or is
                        # about to record itself; taken after `timeout`
                        first = self._orphan.setdefault(i, time.monotonic())
                        if time.monotonic() - first > self.timeout and self._claim(i, "") \
                                and not self._done(i):
                            self._run_one(fn, i, out)
                        continue
                    owner = self.s.get(self._k("owner", i)).decode()
                    if owner == str(self.rank) or not self._stale(int(owner)):
                        continue
                    if self._claim(i, owner) and not self._done(i):
                        self._run_one(fn, i, out)
                time.sleep(poll)
        finally:
            self._stop.set()
            t.join()
        return out

    def gather(self) -> list:
        """Every published result in item order (after run() returned on this rank)."""
        return [pickle.loads(self.s.get(self._k("res", i))) for i in range(self.n)]

"""Per-image data parallelism across GPUs: one process per GPU draws image
indices from one shared host queue (no inter-GPU communication).

Images are independent, so the only shared state is the queue itself and the
host buffers the images live in:

  SharedQueue   a work queue of indices 0..total-1 over a torch.distributed
                key-value Store (the TCPStore of the torchrun rendezvous, so no
                NCCL and no extra service).  take() hands out each index once;
                a worker that dies with indices taken but not done is detected
                by its stale heartbeat and its indices are put back (requeued)
                for the survivors, so every index is done exactly once as long
                as one worker survives.
  HostImagePool a file-backed array of same-shape u8 images that every process
                on the host maps (page cache: one copy in host memory), filled
                cooperatively by the ranks.
  drain()       worker threads of one process: take an index, enhance that
                image through the public GcdrEnhancer API (host buffers in,
                host buffers out), mark it done.

This is the concurrency model the reference offers on one device -- a shared
enhancer whose worker pool serves any number of callers
(src/Sdcb.SimdGcdrNet/GcdrEnhancer.cs:378-432, tested by
tests/Sdcb.SimdGcdrNet.Tests/EngineTests.cs:245-263) -- extended to one such
enhancer per GPU fed by one queue.
"""
from __future__ import annotations

import os
import threading
import time

import numpy as np


class SharedQueue:
    """Indices 0..total-1 handed out once each across processes through `store`.

    Keys (all under `prefix/`): `next` fresh-index counter; `claim/<i>` the rank
    that took i; `done/<i>` set when i is finished; `ndone` finished count;
    `hb/<rank>` heartbeat (time.time() of the rank's latest take, at most every
    `beat_s`); `fin/<rank>` the rank left normally; `rq_len`, `rq_taken`,
    `rq/<slot>` the requeue list; `reaped/<rank>` guards the one-time requeue of
    a dead rank's indices."""

    def __init__(self, store, total: int, rank: int, world: int, prefix: str = "gcdrq", stale_s: float = 10.0,
                 beat_s: float = 0.5):
        self.store, self.total, self.rank, self.world = store, int(total), int(rank), int(world)
        self.p = prefix
        self.stale_s, self.beat_s = stale_s, beat_s
        self._last_beat = 0.0
        self.heartbeat()

    def _k(self, *parts) -> str:
        return "/".join((self.p,) + tuple(str(x) for x in parts))

    def _count(self, key: str) -> int:
        return int(self.store.add(self._k(key), 0))

    def heartbeat(self, force: bool = True):
        now = time.time()
        if force or now - self._last_beat >= self.beat_s:
            self._last_beat = now
            self.store.set(self._k("hb", self.rank), repr(now))

    def _claim(self, i: int) -> int:
        self.store.set(self._k("claim", i), str(self.rank))
        return i

    def take(self, poll_s: float = 0.005):
        """The next index to work on, or None when every index is done."""
        self.heartbeat(force=False)
        n = int(self.store.add(self._k("next"), 1)) - 1
        if n < self.total:
            return self._claim(n)       # two store round trips per fresh index
        # fresh indices exhausted: requeued ones (a dead worker's, put back by reap()), until
        # every index is done
        while True:
            self.heartbeat(force=False)
            rq_len = self._count("rq_len")
            if rq_len and self._count("rq_taken") < rq_len:
                slot = int(self.store.add(self._k("rq_taken"), 1)) - 1
                if slot < rq_len:
                    return self._claim(int(self.store.get(self._k("rq", slot))))
            if self._count("ndone") >= self.total:
                return None
            self.reap()
            time.sleep(poll_s)

    def take_fresh(self):
        """The next fresh index, or None once they are all handed out (never waits: a caller
        that holds taken, unfinished indices may ask for more without waiting on itself)."""
        self.heartbeat(force=False)
        n = int(self.store.add(self._k("next"), 1)) - 1
        return self._claim(n) if n < self.total else None

    def done(self, i: int):
        self.store.set(self._k("done", i), "1")
        self.store.add(self._k("ndone"), 1)

    def finish(self):
        self.store.set(self._k("fin", self.rank), "1")

    def _is_dead(self, r: int, now: float) -> bool:
        if r == self.rank or self.store.check([self._k("fin", r)]):
            return False
        if not self.store.check([self._k("hb", r)]):
            return False            # never started: nothing of its own to requeue
        return now - float(self.store.get(self._k("hb", r)).decode()) > self.stale_s

    def reap(self):
        """Requeues the taken-but-unfinished indices of every rank whose heartbeat is stale."""
        now = time.time()
        for r in range(self.world):
            if not self._is_dead(r, now):
                continue
            # one reaper per dead rank: the first compare-and-set wins, with a token unique to
            # this call (several threads of one survivor, and its later polls, must not
            # requeue the same indices again)
            token = f"{self.rank}:{threading.get_ident()}:{time.monotonic_ns()}"
            if self.store.compare_set(self._k("reaped", r), "", token) != token.encode():
                continue            # reaped already (by another survivor or an earlier call)
            for i in range(self.total):
                if not self.store.check([self._k("claim", i)]) or self.store.check([self._k("done", i)]):
                    continue
                if self.store.get(self._k("claim", i)).decode() != str(r):
                    continue
                slot = int(self.store.add(self._k("rq_len"), 1)) - 1
                self.store.set(self._k("rq", slot), str(i))

    def counts(self) -> tuple:
        """(indices done, indices requeued) over all ranks."""
        return self._count("ndone"), self._count("rq_len")


class HostImagePool:
    """`count` u8 images of `nbytes` each in a file every process of the host maps.

    Rank 0 creates the file; after a barrier every rank opens it.  The mapping is
    shared through the page cache, so the pool lives once in host memory."""

    def __init__(self, path: str, count: int, nbytes: int, create: bool):
        self.path, self.count, self.nbytes = path, int(count), int(nbytes)
        if create:
            with open(path, "wb") as fh:
                fh.truncate(self.count * self.nbytes)
        self.arr = np.memmap(path, dtype=np.uint8, mode="r+", shape=(self.count, self.nbytes))

    def image(self, i: int) -> np.ndarray:
        return self.arr[i]

    def close(self, remove: bool):
        del self.arr
        if remove:
            try:
                os.remove(self.path)
            except OSError:
                pass


def _fill(args):
    path, count, nbytes, idx, make = args
    pool = HostImagePool(path, count, nbytes, create=False)
    for i in idx:
        pool.arr[i] = make(i).reshape(-1)
    pool.arr.flush()
    return len(idx)


def fill_pool(pool: HostImagePool, indices, make, procs: int) -> None:
    """Writes make(i) (a u8 array of pool.nbytes) into pool image i for each index, with
    `procs` worker processes (spawned: safe in a process that has touched the GPU)."""
    indices = list(indices)
    if procs <= 1 or len(indices) <= 1:
        _fill((pool.path, pool.count, pool.nbytes, indices, make))
        return
    import multiprocessing as mp
    chunks = [indices[k::procs] for k in range(procs)]
    with mp.get_context("spawn").Pool(procs) as p:
        p.map(_fill, [(pool.path, pool.count, pool.nbytes, c, make) for c in chunks if c])


def drain(queue: SharedQueue, work, threads: int, batch: int = 1) -> int:
    """Runs `threads` host threads that take indices from `queue` and call work(i)
    (one image each) until every index is done; returns the indices this process did.
    With batch > 1, work receives a list of up to `batch` fresh indices per call (one
    batched enhancement); requeued indices (a dead worker's) come one at a time."""
    did = [0] * threads
    err = []

    def loop(k: int):
        try:
            while True:
                if batch == 1:
                    i = queue.take()
                    if i is None:
                        return
                    work(i)
                    queue.done(i)
                    did[k] += 1
                    continue
                got = []
                while len(got) < batch:
                    i = queue.take_fresh()
                    if i is None:
                        break
                    got.append(i)
                if not got:
                    i = queue.take()    # waits for requeued indices until every index is done
                    if i is None:
                        return
                    got = [i]
                work(got)
                for i in got:
                    queue.done(i)
                did[k] += len(got)
        except BaseException as e:  # surfaced to the caller after the join
            err.append(e)

    th = [threading.Thread(target=loop, args=(k,)) for k in range(threads)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    if err:
        raise err[0]
    queue.finish()
    return sum(did)

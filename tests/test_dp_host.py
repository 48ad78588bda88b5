"""Host logic of the multi-GPU runner (sdcb/gcdrnet_b200/dp.py), on CPU.

The shared queue hands every image index out exactly once across processes;
a worker that dies holding an index is detected by its stale heartbeat and the
index is requeued for the survivors (no GPU: the failure is a host process
that exits while holding work).  The host image pool is one file-backed array
every process maps.
"""
import multiprocessing as mp
import os
import threading

import numpy as np

from sdcb.gcdrnet_b200 import dp


def _store(port=None):
    from torch.distributed import TCPStore
    if port is None:
        return TCPStore("127.0.0.1", 0, is_master=True, wait_for_workers=False)
    return TCPStore("127.0.0.1", port, is_master=False)


def test_queue_hands_out_each_index_once_threads():
    from torch.distributed import HashStore
    total = 200
    q = dp.SharedQueue(HashStore(), total, rank=0, world=1)
    seen = []
    lock = threading.Lock()

    def work(i):
        with lock:
            seen.append(i)

    assert dp.drain(q, work, threads=4) == total
    assert sorted(seen) == list(range(total))
    assert q.counts() == (total, 0)
    assert q.take() is None


def test_batched_drain_hands_out_each_index_once():
    """drain(batch=k): every call gets 1..k fresh indices, every index is done once."""
    from torch.distributed import HashStore
    total = 203
    q = dp.SharedQueue(HashStore(), total, rank=0, world=1)
    seen, sizes = [], []
    lock = threading.Lock()

    def work(ids):
        with lock:
            seen.extend(ids)
            sizes.append(len(ids))

    assert dp.drain(q, work, threads=3, batch=4) == total
    assert sorted(seen) == list(range(total))
    assert max(sizes) == 4 and min(sizes) >= 1
    assert q.counts() == (total, 0)
    assert q.take_fresh() is None and q.take() is None


def _batch_worker(port, rank, world, total, die_after, stale_s, threads):
    st = _store(port)
    q = dp.SharedQueue(st, total, rank=rank, world=world, stale_s=stale_s, beat_s=0.05)
    calls = [0]

    def work(ids):
        if die_after is not None and calls[0] == die_after:
            os._exit(17)                 # dies holding a whole batch (taken, never done)
        for i in ids:
            st.add(f"count/{i}", 1)      # the "enhancement" of image i
        calls[0] += 1

    n = dp.drain(q, work, threads=threads, batch=3)
    st.set(f"did/{rank}", str(n))


def test_batched_drain_requeues_a_dead_workers_batch():
    st = _store()
    total, stale = 60, 0.5
    ctx = mp.get_context("spawn")
    dying = ctx.Process(target=_batch_worker, args=(st.port, 0, 2, total, 2, stale, 1))
    dying.start()
    dying.join(60)
    assert dying.exitcode == 17
    # the survivor drains the fresh indices, then redoes the dead worker's held batch
    alive = ctx.Process(target=_batch_worker, args=(st.port, 1, 2, total, None, stale, 2))
    alive.start()
    alive.join(60)
    assert alive.exitcode == 0
    counts = [int(st.add(f"count/{i}", 0)) for i in range(total)]
    assert counts == [1] * total, "every index enhanced exactly once"
    assert int(st.add("gcdrq/rq_len", 0)) == 3, "the held batch of three was requeued"
    assert int(st.get("did/1")) == total - 6


def _worker(port, rank, world, total, die_after, stale_s):
    st = _store(port)
    q = dp.SharedQueue(st, total, rank=rank, world=world, stale_s=stale_s, beat_s=0.05)
    n = 0
    while True:
        i = q.take()
        if i is None:
            break
        if die_after is not None and n == die_after:
            os._exit(17)                 # dies holding index i (taken, never done)
        st.add(f"count/{i}", 1)          # the "enhancement" of image i
        q.done(i)
        n += 1
    q.finish()
    st.set(f"did/{rank}", str(n))


def test_queue_requeues_the_work_of_a_dead_worker():
    st = _store()
    total, stale = 60, 0.5
    ctx = mp.get_context("spawn")
    dying = ctx.Process(target=_worker, args=(st.port, 0, 2, total, 5, stale))
    dying.start()
    dying.join(60)
    assert dying.exitcode == 17
    # the survivor drains the rest, notices the stale heartbeat and redoes the held index
    alive = ctx.Process(target=_worker, args=(st.port, 1, 2, total, None, stale))
    alive.start()
    alive.join(60)
    assert alive.exitcode == 0
    counts = [int(st.add(f"count/{i}", 0)) for i in range(total)]
    assert counts == [1] * total, "every index enhanced exactly once"
    assert int(st.add("gcdrq/rq_len", 0)) == 1
    assert int(st.get("did/1")) == total - 5


def test_queue_two_live_workers_share_the_work():
    st = _store()
    total = 80
    ctx = mp.get_context("spawn")
    ps = [ctx.Process(target=_worker, args=(st.port, r, 2, total, None, 5.0)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
    assert [p.exitcode for p in ps] == [0, 0]
    assert [int(st.add(f"count/{i}", 0)) for i in range(total)] == [1] * total
    assert int(st.get("did/0")) + int(st.get("did/1")) == total


def test_host_image_pool_is_shared_between_processes(tmp_path):
    from sdcb.gcdrnet_b200 import synth
    path = str(tmp_path / "pool.u8")
    w, h = 64, 48
    pool = dp.HostImagePool(path, 6, w * h * 3, create=True)
    dp.fill_pool(pool, range(6), synth.DocumentMaker(w, h), procs=2)
    for i in range(6):
        assert np.array_equal(pool.image(i), synth.document(w, h, seed=i).reshape(-1))
    pool.close(remove=True)
    assert not os.path.exists(path)

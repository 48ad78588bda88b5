"""Host logic of the multi-GPU bench on CPU: world_size-2 `gloo` ranks.

The path shards by image (no data-path collective, no NCCL): the ranks meet
only on the host -- the max/min over ranks of the timed region, which sets the
whole-job rate, and the shared image queue carried by the rendezvous store.
These tests run that logic as two CPU processes.
"""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        local_ms = 100.0 + 25.0 * rank            # rank 1 is the slower one
        total_ms = bench.max_over_ranks(local_ms, dist)
        start = bench.min_over_ranks(10.0 + rank, dist)
        seeds = bench.rank_seeds(rank, 4)
        gathered = [None] * world
        dist.all_gather_object(gathered, seeds)
        rate = bench.whole_job_rate(world, 10, total_ms / 1000.0)
        # the c3 drain: both ranks take image indices from one queue on the rendezvous store
        import time
        from sdcb.gcdrnet_b200 import dp
        store = dist.distributed_c10d._get_default_store()
        q = dp.SharedQueue(store, 40, rank, world, prefix="c3")
        mine = []

        def work(i):
            time.sleep(0.002 * (1 + rank))     # rank 1 is slower: it should take fewer
            mine.append(i)

        did = dp.drain(q, work, threads=2)
        per_rank = bench.gather_ints(did, dist, world)
        taken = [None] * world
        dist.all_gather_object(taken, sorted(mine))
        with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as fh:
            fh.write(repr((total_ms, start, gathered, rate, per_rank, taken)))
    finally:
        dist.destroy_process_group()


def test_two_rank_max_and_rate(tmp_path):
    world = 2
    mp.spawn(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    res = [eval(open(tmp_path / f"r{r}.txt").read()) for r in range(world)]
    for total_ms, start, gathered, rate, per_rank, taken in res:
        assert total_ms == 125.0, "every rank must see the slowest rank's time"
        assert start == 10.0, "the job starts at the earliest rank's start"
        assert rate == pytest.approx(2 * 10 / 0.125)
        flat = [s for g in gathered for s in g]
        assert len(set(flat)) == len(flat), "ranks must enhance disjoint images"
        assert sum(per_rank) == 40 and min(per_rank) > 0
        assert sorted(taken[0] + taken[1]) == list(range(40)), "each queued image taken exactly once"


def test_single_rank_is_identity():
    assert bench.max_over_ranks(3.5) == 3.5
    assert bench.min_over_ranks(3.5) == 3.5
    assert bench.gather_ints(7) == [7]
    assert bench.whole_job_rate(1, 20, 2.0) == 10.0
    assert bench.rank_seeds(0, 3) == [0, 1, 2]


def test_reference_arm_other_ranks_exit_without_work(monkeypatch, capsys):
    monkeypatch.setenv("RANK", "1")

    class A:
        gpus, steps, warmup = 2, 3, 3
    assert bench.run_reference(A()) == 0
    assert capsys.readouterr().out == ""

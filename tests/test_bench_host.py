"""Host logic of the multi-GPU bench on CPU: world_size-2 `gloo` ranks.

The path shards by image (no data-path collective); the only collective is
the max over ranks of the timed region, which sets the whole-job rate.  These
tests run that logic as two CPU processes.
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
        total_ms = bench.max_over_ranks(local_ms, dist, "cpu")
        seeds = bench.rank_seeds(rank, 4)
        gathered = [None] * world
        dist.all_gather_object(gathered, seeds)
        rate = bench.whole_job_rate(world, 10, total_ms / 1000.0)
        with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as fh:
            fh.write(repr((total_ms, gathered, rate)))
    finally:
        dist.destroy_process_group()


def test_two_rank_max_and_rate(tmp_path):
    world = 2
    mp.spawn(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    res = [eval(open(tmp_path / f"r{r}.txt").read()) for r in range(world)]
    for total_ms, gathered, rate in res:
        assert total_ms == 125.0, "every rank must see the slowest rank's time"
        assert rate == pytest.approx(2 * 10 / 0.125)
        flat = [s for g in gathered for s in g]
        assert len(set(flat)) == len(flat), "ranks must enhance disjoint images"


def test_single_rank_is_identity():
    assert bench.max_over_ranks(3.5) == 3.5
    assert bench.whole_job_rate(1, 20, 2.0) == 10.0
    assert bench.rank_seeds(0, 3) == [0, 1, 2]


def test_reference_arm_other_ranks_exit_without_work(monkeypatch, capsys):
    monkeypatch.setenv("RANK", "1")

    class A:
        gpus, steps, warmup = 2, 3, 3
    assert bench.run_reference(A()) == 0
    assert capsys.readouterr().out == ""

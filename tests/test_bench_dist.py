"""Multi-rank host logic of bench.py on CPU with the gloo backend
(world_size 2): max-over-ranks timing, whole-job aggregation and the
rank-0-only reference arm."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        my_ms = 2.0 + rank                       # rank 1 is slower
        slowest = bench.max_over_ranks(my_ms, world)
        rate = bench.whole_job_rate(1e12, world, slowest)
        bench.barrier(world)
        out[rank] = (slowest, rate)
    finally:
        dist.destroy_process_group()


def test_two_rank_max_and_whole_job_rate():
    world = 2
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    assert res[0] == res[1]
    slowest, rate = res[0]
    assert slowest == 3.0
    assert rate == pytest.approx(2 * 1e12 / 3e-3)


def test_reference_arm_runs_on_rank_zero_only(capsys, monkeypatch):
    monkeypatch.setenv("RANK", "1")
    rc = bench.main(["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0"])
    assert rc == 0
    assert capsys.readouterr().out == ""

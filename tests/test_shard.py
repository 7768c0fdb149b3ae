"""Multi-GPU partitioning (glaucis_b200/shard.py) on CPU: the expert-group
row partition and its per-rank group sizes, the head partition, and the row
all-gather across two gloo ranks (equal and padded slabs)."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from glaucis_b200 import configs, shard


def _check_partition(sizes, world):
    parts = shard.gmm_partition(sizes, world)
    off = np.concatenate([[0], np.cumsum(sizes)])
    assert parts[0].r0 == 0 and parts[-1].r1 == off[-1]
    for a, b in zip(parts, parts[1:]):
        assert a.r1 == b.r0
    for p in parts:
        assert p.r0 % 128 == 0 or p.r0 == off[-1]
        assert int(p.sizes.sum()) == p.rows
        if p.rows:
            # the local groups cover exactly [r0, r1) in order
            assert off[p.g0] <= p.r0 < off[p.g0 + 1] or sizes[p.g0] == 0
            assert off[p.g1 - 1] < p.r1 <= off[p.g1]
    counts = [p.rows for p in parts]
    assert max(counts) - min(counts) <= 128 * 2
    return parts


def test_gmm_partition_dense_expert_and_moe():
    for name, world in (("gmm_dense_expert", 8), ("gmm_dense_expert", 2), ("gmm_moe_up", 4),
                        ("gmm_small", 2)):
        cfg = configs.GMM_CONFIGS[name]
        sizes = configs.group_sizes(cfg.routing, cfg.G, cfg.M, seed=0)
        parts = _check_partition(np.asarray(sizes), world)
        if name == "gmm_dense_expert" and world == 8:
            assert [p.rows for p in parts] == [8192] * 8


def test_gmm_partition_edge_cases():
    _check_partition(np.array([0, 0, 300, 0, 5, 0]), 2)     # empty groups, ragged tail
    parts = shard.gmm_partition(np.array([100]), 4)          # fewer tiles than ranks
    assert sum(p.rows for p in parts) == 100 and parts[-1].r1 == 100
    assert [p.rows for p in parts].count(0) >= 2


def test_gla_head_partition():
    for H, w in ((32, 8), (32, 3), (16, 2), (5, 4)):
        parts = shard.gla_head_partition(H, w)
        assert [h for r in parts for h in r] == list(range(H))
        assert max(len(r) for r in parts) - min(len(r) for r in parts) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        for counts in ([3, 3], [5, 2]):
            local = torch.arange(counts[rank] * 4, dtype=torch.float32).reshape(-1, 4) + 100 * rank
            full = torch.empty((sum(counts), 4))
            shard.all_gather_rows(local, counts, full)
            out[(rank, tuple(counts))] = full.numpy().tolist()
    finally:
        dist.destroy_process_group()


def test_all_gather_rows_two_gloo_ranks():
    world = 2
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
        res = dict(out)
    for counts in ([3, 3], [5, 2]):
        want = np.concatenate([np.arange(counts[r] * 4, dtype=np.float32).reshape(-1, 4) + 100 * r
                               for r in range(world)])
        for r in range(world):
            np.testing.assert_array_equal(np.asarray(res[(r, tuple(counts))]), want)


def test_ring_order_spreads_the_first_peer_store():
    ptrs = [100, 101, 102, 103]
    orders = [shard.ring_order(ptrs, r) for r in range(4)]
    assert orders[0] == [100, 101, 102, 103] and orders[2] == [102, 103, 100, 101]
    for k in range(4):  # at every position the four ranks target four different buffers
        assert sorted(o[k] for o in orders) == ptrs

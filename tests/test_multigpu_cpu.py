"""CPU: the multi-GPU host logic with world-size-2 gloo process groups.

Sharding covers every head exactly once, per-rank seeds differ, and the job
time is the max over ranks (what bench.py reports for N > 1 under torchrun).
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tilemix_b200 import sharding


def test_shard_heads_partition():
    for total in (0, 1, 7, 256, 1000):
        for world in (1, 2, 3, 8):
            covered = []
            for rank in range(world):
                start, count = sharding.shard_heads(total, world, rank)
                covered.extend(range(start, start + count))
            assert covered == list(range(total))
            counts = [sharding.shard_heads(total, world, r)[1] for r in range(world)]
            assert max(counts) - min(counts) <= 1
    with pytest.raises(ValueError):
        sharding.shard_heads(10, 2, 2)


def test_rank_seeds_distinct():
    seeds = {sharding.rank_seed(2, r) for r in range(8)}
    assert len(seeds) == 8 and sharding.rank_seed(2, 0) == 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # each rank's "device time" and its head shard of a 256-head batch
        my_time = 1.5 + rank
        start, count = sharding.shard_heads(256, world, rank)
        job_time = sharding.max_over_ranks(my_time, world)
        heads = sharding.sum_over_ranks(count, world)
        dist.barrier()
        results[rank] = (job_time, heads, start, count)
    finally:
        dist.destroy_process_group()


def test_gloo_world2_max_and_shards():
    world = 2
    port = _free_port()
    manager = mp.get_context("spawn").Manager()   # no fork of this (multi-threaded) process
    results = manager.dict()
    mp.spawn(_worker, args=(world, port, results), nprocs=world, join=True)
    assert results[0][0] == results[1][0] == 2.5          # slowest rank
    assert results[0][1] == results[1][1] == 256          # every head once
    assert results[0][2:] == (0, 128) and results[1][2:] == (128, 128)

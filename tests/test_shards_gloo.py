"""The multi-GPU host logic (qwenscriber_b200.shards) on two gloo ranks on the
CPU: streams shard by stream with no exchange, every rank derives the same
global prefix lengths, and timings reduce to the slowest rank."""

import os
import socket

import pytest
import torch.multiprocessing as mp

from qwenscriber_b200 import shards, synthetic


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, out):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        w = synthetic.workloads()["cfg4_1p7b_q4_s64_long"]
        ids = list(shards.shard(w.streams * world, world, rank))
        lengths = synthetic.prefix_lengths(w, world, rank)
        slowest = shards.max_over_ranks(1.0 + rank)  # a device time that differs per rank
        got = [None] * world
        dist.all_gather_object(got, (ids, lengths))
        out[rank] = (got, slowest, shards.aggregate_rate(w.streams, world, slowest))
    finally:
        dist.destroy_process_group()


def test_shard_ranges_are_disjoint_and_cover():
    for total, world in ((512, 8), (64, 1), (10, 3)):
        seen = [g for r in range(world) for g in shards.shard(total, world, r)]
        assert seen == list(range(total))
    with pytest.raises(ValueError):
        shards.shard(8, 2, 2)


def test_prefix_lengths_do_not_depend_on_the_gpu_count():
    w = synthetic.workloads()["cfg4_1p7b_q4_s64_long"]
    one = synthetic.prefix_lengths(w)
    eight = [x for r in range(8) for x in synthetic.prefix_lengths(w, 8, r)]
    assert eight[:64] == one and len(eight) == 512
    assert all(2048 <= x <= 3584 for x in eight)


def test_max_over_ranks_without_a_group_is_the_value():
    assert shards.max_over_ranks(3.5) == 3.5


def test_two_gloo_ranks():
    world, port = 2, _free_port()
    with mp.Manager() as manager:
        out = manager.dict()
        mp.start_processes(_rank, args=(world, port, out), nprocs=world, join=True, start_method="spawn")
        results = dict(out)
    w = synthetic.workloads()["cfg4_1p7b_q4_s64_long"]
    assert sorted(results) == [0, 1]
    for rank in range(world):
        gathered, slowest, rate = results[rank]
        assert slowest == 2.0  # the max over ranks
        assert rate == w.streams * world / 2.0
        ids = [g for r_ids, _ in gathered for g in r_ids]
        assert ids == list(range(w.streams * world))  # disjoint, covering, in rank order
        lengths = [x for _, r_len in gathered for x in r_len]
        assert lengths == shards.prefix_lengths(2048, 3584, w.seed, w.streams * world)

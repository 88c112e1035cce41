"""World-size-2 ``gloo`` tests (CPU) of the multi-GPU host logic: sequence
sharding, seeded per-sequence contexts, max-over-ranks timing and the
aggregate throughput of the sequence-sharded batched decode."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flux_b200 import sharding


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, queue) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        shard = sharding.sequence_shard(128, world, rank)
        lengths, tokens = sharding.shard_contexts(7, shard, 512, 4096)
        my_ms = [10.0 + rank, 3.0 * (world - rank)]
        worst = sharding.max_over_ranks(my_ms)
        total = sharding.aggregate_tokens_per_s(len(shard) * 256, world, worst[0])
        queue.put((rank, list(shard), lengths, tokens, worst, total))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_and_timing():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, shard, lengths, tokens, worst, total = queue.get(timeout=120)
        results[rank] = (shard, lengths, tokens, worst, total)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # disjoint contiguous shards covering all sequences
    assert results[0][0] == list(range(0, 64)) and results[1][0] == list(range(64, 128))
    # every rank sees the same max-over-ranks times and aggregate
    assert results[0][3] == results[1][3] == [11.0, 6.0]
    assert results[0][4] == results[1][4] == pytest.approx(2 * 64 * 256 / 11e-3)
    # a sequence's context does not depend on the world size
    single, _ = sharding.shard_contexts(7, sharding.sequence_shard(128, 1, 0), 512, 4096)
    assert results[0][1] + results[1][1] == single
    assert all(512 <= n <= 4096 for n in single)


def test_sharding_rejects_uneven_and_bad_rank():
    with pytest.raises(ValueError):
        sharding.sequence_shard(100, 3, 0)
    with pytest.raises(ValueError):
        sharding.sequence_shard(64, 2, 2)
    assert sharding.max_over_ranks([1.0, 2.0]) == [1.0, 2.0]  # no process group: identity

"""Multi-process host logic of the N-GPU bench on CPU: gloo, world size 2."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from transformer_opt.sharding import gather_stats, max_over_ranks, shard_range


@pytest.mark.parametrize("total,world", [(8, 1), (8, 2), (8, 3), (512, 8), (4, 8), (1, 2)])
def test_shard_range_partitions_exactly(total, world):
    spans = [shard_range(total, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == total
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dev = torch.device("cpu")
        start, stop = shard_range(10, world, rank)
        stats = gather_stats([float(rank), float(stop - start)], dev)
        worst = max_over_ranks(1.5 * (rank + 1), dev)
        queue.put((rank, stats, worst))
    finally:
        dist.destroy_process_group()


def test_two_rank_gather_and_max_over_ranks():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict()
    for _ in procs:
        rank, stats, worst = queue.get(timeout=120)
        results[rank] = (stats, worst)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in (0, 1):
        stats, worst = results[rank]
        assert stats == [[0.0, 5.0], [1.0, 5.0]]
        assert worst == 3.0


def _gather_worker(rank, world, port, queue):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        total = 11  # uneven shards: 6 + 5 sequences
        full = torch.arange(total * 3 * 4, dtype=torch.float32).view(total, 3, 4)
        start, stop = shard_range(total, world, rank)
        indices = bench.sample_indices("C5", total)
        sample = bench.gather_sample(full[start:stop], start, indices, world, torch.device("cpu"))
        queue.put((rank, indices, None if sample is None else sample.tolist()))
    finally:
        dist.destroy_process_group()


def test_output_sample_gathers_the_global_sequences_to_rank_0():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, indices, sample = queue.get(timeout=120)
        results[rank] = (indices, sample)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    indices, sample = results[0]
    full = torch.arange(11 * 3 * 4, dtype=torch.float32).view(11, 3, 4)
    assert indices == [0, 1, 3, 4, 6, 7, 9, 10]  # 8 spread over 11 sequences
    assert torch.equal(torch.tensor(sample), full[indices])
    assert results[1][1] is None  # only rank 0 receives the sample

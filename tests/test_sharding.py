"""Sharding helpers, including the N>1 all-gather path on world_size-2 gloo
ranks (CPU, no GPU needed)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ninetoothed_b200.sharding import gather_rows, shard_range, shard_rows


@pytest.mark.parametrize("total, world", [(16384, 1), (16384, 8), (10, 3), (3, 4), (0, 2)])
def test_shard_range_partitions_exactly(total, world):
    ranges = [shard_range(total, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == total
    for (a, b), (c, d) in zip(ranges, ranges[1:]):
        assert b == c and b >= a
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, rows, cols, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = torch.arange(rows * cols, dtype=torch.float32).reshape(rows, cols)
        mine = shard_rows(full, rank, world)
        # each rank "computes" its shard (here: a row-wise softmax on CPU)
        out = torch.softmax(mine, dim=-1)
        gathered = gather_rows(out, rows)
        results[rank] = bool(torch.equal(gathered, torch.softmax(full, dim=-1)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rows", [8, 7])
def test_gather_rows_two_gloo_ranks(rows):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, rows, 5, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert dict(results) == {0: True, 1: True}

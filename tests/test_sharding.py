"""Sharding helpers, including the N>1 all-gather path on world_size-2 gloo
ranks (CPU, no GPU needed)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ninetoothed_b200.sharding import gather_rows, shard_pairs, shard_range, shard_rows


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


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_pairs_views_cover_every_batch_head_pair_once(world):
    t = torch.arange(4 * 32 * 3 * 2, dtype=torch.float32).reshape(4, 32, 3, 2)
    views = [shard_pairs(t, r, world) for r in range(world)]
    assert all(v.dim() == 4 and v.shape[0] == 1 for v in views)
    assert torch.equal(torch.cat([v[0] for v in views]), t.reshape(128, 3, 2))
    views[-1].fill_(-1)  # views, not copies
    assert bool((t.reshape(128, 3, 2)[-views[-1].shape[1]:] == -1).all())


def test_shard_pairs_refuses_a_layout_that_needs_a_copy():
    t = torch.zeros(4, 32, 8, 2).transpose(0, 1)
    with pytest.raises(ValueError):
        shard_pairs(t, 0, 2)


def _cpu_kernels(monkeypatch_target):
    """CPU stand-ins for the B200 kernels, so the sharded entry points' split
    and gather logic runs on gloo ranks without a GPU."""
    import torch.nn.functional as F

    from ninetoothed_b200 import programs

    programs.softmax_kernel = lambda x, y, BLOCK_SIZE=None: y.copy_(torch.softmax(x, -1))
    programs.matmul_kernel = lambda a, b, out: out.copy_(a @ b)
    programs.addmm_kernel = lambda i, a, b, beta, alpha, out: out.copy_(beta * i + alpha * (a @ b))
    programs.attention_kernel = lambda q, k, v, causal, o: o.copy_(
        F.scaled_dot_product_attention(q, k, v, is_causal=bool(causal), scale=1.0))
    programs.conv2d_kernel = lambda x, w, y, padding_h=0, padding_w=0: y.copy_(
        F.conv2d(x, w, padding=(padding_h, padding_w)))
    return programs


def _programs_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ninetoothed_b200 import sharding

        _cpu_kernels(None)
        g = torch.Generator().manual_seed(0)  # every rank holds the same whole logical inputs
        ok = {}
        x = torch.randn(13, 40, generator=g)
        y = torch.empty_like(x)
        mine = sharding.softmax_shard(x, y, rank, world)
        ok["softmax"] = torch.allclose(gather_rows(mine.contiguous(), 13), torch.softmax(x, -1))
        a, b, i = torch.randn(11, 6, generator=g), torch.randn(6, 5, generator=g), torch.randn(11, 5, generator=g)
        out = torch.empty(11, 5)
        mine = sharding.matmul_shard(a, b, out, rank, world)
        ok["matmul"] = torch.allclose(gather_rows(mine.contiguous(), 11), a @ b, atol=1e-6)
        mine = sharding.addmm_shard(i, a, b, 0.5, 2.0, out, rank, world)
        ok["addmm"] = torch.allclose(gather_rows(mine.contiguous(), 11), 0.5 * i + 2.0 * (a @ b), atol=1e-5)
        q, k, v = (torch.randn(2, 3, 7, 4, generator=g) for _ in range(3))
        o = torch.empty_like(q)
        mine = sharding.attention_shard(q, k, v, True, o, rank, world)
        import torch.nn.functional as F

        full = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=1.0).reshape(6, 7, 4)
        ok["attention"] = torch.allclose(gather_rows(mine[0].contiguous(), 6), full, atol=1e-6)
        xi, w = torch.randn(5, 3, 6, 6, generator=g), torch.randn(4, 3, 3, 3, generator=g)
        yi = torch.empty(5, 4, 6, 6)
        mine = sharding.conv2d_shard(xi, w, yi, 1, rank, world)
        ok["conv2d"] = torch.allclose(gather_rows(mine.contiguous(), 5), F.conv2d(xi, w, padding=1), atol=1e-5)
        results[rank] = ok
    finally:
        dist.destroy_process_group()


def test_sharded_programs_on_two_gloo_ranks():
    """Each rank runs its part of softmax / matmul / addmm / attention / conv2d
    through the sharded entry points (CPU stand-ins for the kernels); the
    all-gathered shards equal the whole computation."""
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_programs_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs)
    for rank in (0, 1):
        assert all(results[rank].values()), results[rank]

"""Work partitioning across the GPUs of one node (one process per GPU).

Every benchmarked program shards with no reduction: matmul/addmm by output rows
(each rank holds its rows of A/bias and a replica of B), attention by
(batch x head) pairs, conv2d/max_pool2d by images, softmax by rows.  The only
collective is an optional all-gather of the output shards over NCCL, which
`gather_rows` performs when a caller wants the full result on every rank.
"""

import torch
import torch.distributed as dist


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of `rank`'s contiguous share of `total` units; the first
    `total % world` ranks take one extra unit."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad shard request: total={total} rank={rank} world={world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_rows(tensor: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    """This rank's slice of `tensor` along `dim` (a view, no copy)."""
    start, stop = shard_range(tensor.shape[dim], rank, world)
    return tensor.narrow(dim, start, stop - start)


def gather_rows(shard: torch.Tensor, total_rows: int, group=None) -> torch.Tensor:
    """All-gather equal or near-equal row shards into the full tensor on every
    rank.  Uneven shards are padded to the largest share for the collective and
    trimmed afterwards."""
    world = dist.get_world_size(group)
    largest = shard_range(total_rows, 0, world)[1]
    padded = shard.new_zeros((largest, *shard.shape[1:]))
    padded[: shard.shape[0]] = shard
    out = shard.new_empty((largest * world, *shard.shape[1:]))
    dist.all_gather_into_tensor(out, padded.contiguous(), group=group)
    pieces = []
    for r in range(world):
        start, stop = shard_range(total_rows, r, world)
        pieces.append(out[r * largest : r * largest + (stop - start)])
    return torch.cat(pieces, dim=0)

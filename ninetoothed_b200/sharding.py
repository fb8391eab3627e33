"""Work partitioning of the operator programs across the GPUs of one node.

One process per GPU; every program splits with no reduction, so the ranks
never exchange data on the compute path:

  softmax          rows of the [rows, cols] input and output;
  matmul / addmm   rows of A (and of the addmm input and the output), B
                   replicated on every rank;
  attention        (batch, head) pairs of q, k, v and o;
  conv2d,          images of the input and output (the filter replicated);
  max_pool2d

Each `*_shard` function takes the whole logical tensors of one call (views
on this rank's device) and runs the B200 kernel on this rank's part of them,
writing this rank's part of the output; `shard_*` return the views.  The only
collective is the optional all-gather of output shards over NCCL
(`gather_rows`) for a caller that wants the whole result on every rank.
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


def shard_pairs(tensor: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's (batch, head) pairs of a [B, H, S, D] tensor as a
    [1, pairs, S, D] view.  Batch and head must merge into one dimension
    without a copy (true for contiguous tensors); a copy would detach an
    output from the caller's tensor, so it is refused."""
    if tensor.dim() != 4:
        raise ValueError("shard_pairs takes a [batch, heads, seq, head_dim] tensor")
    b, h = tensor.shape[:2]
    if b > 1 and tensor.stride(0) != h * tensor.stride(1):
        raise ValueError("batch and head dimensions do not merge into one without a copy")
    merged = tensor.as_strided((b * h, *tensor.shape[2:]), (tensor.stride(1), *tensor.stride()[2:]))
    return shard_rows(merged, rank, world).unsqueeze(0)


# ---------------------------------------------------------------- programs, split by rank
def softmax_shard(input, output, rank, world):
    """Row softmax of this rank's rows (tests/test_softmax.py:10-27)."""
    from ninetoothed_b200 import programs

    x, y = shard_rows(input, rank, world), shard_rows(output, rank, world)
    if x.shape[0]:
        programs.softmax_kernel(x, y, BLOCK_SIZE=input.shape[-1])
    return y


def matmul_shard(lhs, rhs, output, rank, world):
    """This rank's rows of lhs @ rhs (tests/test_matmul.py:14-47)."""
    from ninetoothed_b200 import programs

    a, out = shard_rows(lhs, rank, world), shard_rows(output, rank, world)
    if a.shape[0]:
        programs.matmul_kernel(a, rhs, out)
    return out


def addmm_shard(input, mat1, mat2, beta, alpha, output, rank, world):
    """This rank's rows of beta * input + alpha * mat1 @ mat2
    (tests/test_addmm.py:13-38)."""
    from ninetoothed_b200 import programs

    i, a, out = (shard_rows(t, rank, world) for t in (input, mat1, output))
    if a.shape[0]:
        programs.addmm_kernel(i, a, mat2, beta, alpha, out)
    return out


def attention_shard(q, k, v, is_causal, o, rank, world):
    """Attention of this rank's (batch, head) pairs (tests/test_attention.py:14-96)."""
    from ninetoothed_b200 import programs

    qs, ks, vs, os_ = (shard_pairs(t, rank, world) for t in (q, k, v, o))
    if qs.shape[1]:
        programs.attention_kernel(qs, ks, vs, is_causal, os_)
    return os_


def conv2d_shard(input, filter, output, padding, rank, world):
    """conv2d of this rank's images (tests/test_conv2d.py:14-49)."""
    from ninetoothed_b200 import programs

    ph, pw = (padding, padding) if isinstance(padding, int) else padding
    x, y = shard_rows(input, rank, world), shard_rows(output, rank, world)
    if x.shape[0]:
        programs.conv2d_kernel(x, filter, y, padding_h=ph, padding_w=pw)
    return y


def max_pool2d_shard(input, output, window, stride, padding, rank, world):
    """max_pool2d of this rank's images (tests/test_max_pool2d.py:13-36 with
    stride and padding)."""
    from ninetoothed_b200 import programs

    x, y = shard_rows(input, rank, world), shard_rows(output, rank, world)
    if x.shape[0]:
        programs.max_pool2d_kernels[False](x, y, WINDOW_HEIGHT=window[0], WINDOW_WIDTH=window[1],
                                           STRIDE_HEIGHT=stride[0], STRIDE_WIDTH=stride[1],
                                           PADDING_HEIGHT=padding[0], PADDING_WIDTH=padding[1])
    return y


# ---------------------------------------------------------------- optional gather
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

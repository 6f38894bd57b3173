"""Column-parallel quantized matmul over several GPUs (one process per GPU).

The reference quantizes each output column independently (one scale per
column, src/quantization/quantization.cpp:141-159) and stores a column's codes
contiguously (quantization.cpp:155), so a weight splits into column shards
with no communication: rank r owns columns [begin_r, end_r), computes
y[:, begin_r:end_r] = matmul(x, W[:, begin_r:end_r]) with the same
activation codes as every other rank (the per-row quantizer depends only on
x), and the shards are joined with one NCCL all-gather only when the caller
needs the full output.  Results are bit-identical to the single-GPU matmul.
"""
from __future__ import annotations


def column_ranges(n_cols: int, world: int):
    """Contiguous, balanced column shards: the first n_cols % world ranks get
    one extra column."""
    if world < 1:
        raise ValueError("world must be >= 1")
    if n_cols < world:
        raise ValueError(f"cannot split {n_cols} columns over {world} ranks")
    base, extra = divmod(n_cols, world)
    out, c = [], 0
    for r in range(world):
        w = base + (1 if r < extra else 0)
        out.append((c, c + w))
        c += w
    return out


def shard_weight(weight, rank: int, world: int):
    """This rank's column shard of a QuantizedMatrix (device to device)."""
    b, e = column_ranges(weight.cols(), world)[rank]
    return weight.slice_cols(b, e)


def assemble_columns(blocks, ranges, out=None):
    """Join gathered per-rank blocks [M, n_r] into [M, N] (column order of
    ``ranges``)."""
    import torch

    M = blocks[0].shape[0]
    N = ranges[-1][1]
    if out is None:
        out = torch.empty((M, N), dtype=blocks[0].dtype, device=blocks[0].device)
    for (b, e), blk in zip(ranges, blocks):
        out[:, b:e].copy_(blk)
    return out


def sharded_matmul(x, weight_shard, n_cols: int, group=None, gather: bool = True, matmul_fn=None, bias_shard=None):
    """y = matmul(x, W) with W column-sharded over the process group.

    ``weight_shard`` is this rank's shard (see :func:`shard_weight`),
    ``n_cols`` the full column count.  With ``gather`` every rank returns the
    full [M, n_cols] output (one all-gather), otherwise its own block.
    ``matmul_fn`` defaults to :func:`zyron_b200.quantization.matmul`.
    """
    import torch
    import torch.distributed as dist

    if matmul_fn is None:
        from .quantization import matmul as matmul_fn
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    ranges = column_ranges(n_cols, world)
    local = matmul_fn(x, weight_shard, bias=bias_shard) if bias_shard is not None else matmul_fn(x, weight_shard)
    b, e = ranges[rank]
    if local.shape[-1] != e - b:
        raise ValueError(f"rank {rank}: shard has {local.shape[-1]} columns, expected {e - b}")
    if not gather or world == 1:
        return local
    widths = [e - b for b, e in ranges]
    M = local.shape[0]
    wmax = max(widths)
    send = local.contiguous()
    if send.shape[1] != wmax:  # uneven split: pad this block to the widest shard
        send = torch.nn.functional.pad(send, (0, wmax - send.shape[1]))
    buf = torch.empty((world * M, wmax), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, send, group=group)
    blocks = [blk[:, :w] for blk, w in zip(buf.view(world, M, wmax).unbind(0), widths)]
    return assemble_columns(blocks, ranges)

"""Host-side partitioning for running the matmul path on several GPUs of one node.

One process per GPU (torchrun), ``torch.distributed`` for the plumbing (NCCL over NVLink on
the GPUs; gloo works the same way on CPU tensors, which is how the logic is tested).

- Column sharding (lm_head N=51200, fc1 N=8192): in the GGUF [N][K] layout an output column
  is a weight row, so rank r owns the contiguous row range ``column_shard(N, world, r)`` of W
  (a plain byte range of the packed blocks: no repacking) and produces those outputs; the
  full vector is rebuilt with one all-gather.
- Batch sharding (SigLIP images, decode sequences): rank r owns ``batch_shard(B, world, r)``;
  the work is independent and needs no exchange.
"""
from __future__ import annotations


def column_shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of the n output columns (= GGUF weight rows) owned by `rank`.  The first
    n % world ranks get one extra column, so shard sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_sizes(n: int, world: int) -> list[int]:
    return [b - a for a, b in (column_shard(n, world, r) for r in range(world))]


def batch_shard(b: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of the b independent items (images, sequences) owned by `rank`."""
    return column_shard(b, world, rank)


def weight_row_bytes_range(n: int, row_bytes: int, world: int, rank: int) -> tuple[int, int]:
    """Byte range of rank's rows inside a packed [N][row_bytes] weight."""
    a, b = column_shard(n, world, rank)
    return a * row_bytes, b * row_bytes


def gather_columns(local, n: int, group=None):
    """All-gather the ranks' column shards (1-D tensors) into the full length-n vector, in
    rank order.  Uses the single-buffer collective when the shards are equal."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    sizes = shard_sizes(n, world)
    if local.numel() != sizes[dist.get_rank(group)]:
        raise ValueError(f"local shard has {local.numel()} values, expected {sizes[dist.get_rank(group)]}")
    width = max(sizes)
    if len(set(sizes)) == 1:
        out = torch.empty(n, dtype=local.dtype, device=local.device)
        dist.all_gather(list(out.split(sizes)), local.contiguous(), group=group)
        return out
    # Unequal shards (n % world != 0): pad every shard to the widest, gather, then trim.
    padded = torch.zeros(width, dtype=local.dtype, device=local.device)
    padded[: local.numel()] = local
    slots = torch.empty(world * width, dtype=local.dtype, device=local.device)
    dist.all_gather(list(slots.split(width)), padded, group=group)
    return torch.cat([slots[r * width: r * width + sizes[r]] for r in range(world)])


def combine_argmax(pairs: list[tuple[int, float]], n: int, world: int) -> int:
    """The global greedy token from the ranks' (local index, value) argmax results over their
    column shards (in rank order): the larger value wins and, between equal values, the
    smaller global index (the lower rank), which is the reference's first maximum.  If no
    shard saw a value above -1e30 the answer is index 0, as in the reference's scan."""
    best_i, best_v = 0, -1e30
    for r, (i, v) in enumerate(pairs):
        g = column_shard(n, world, r)[0] + i
        if v > best_v:
            best_i, best_v = g, v
    return best_i


def combine_argmax_device(slots, offsets):
    """combine_argmax on the device, with no host round trip: `slots` holds the ranks'
    all-gathered (index, fp32 value bits) int32 pairs in rank order, `offsets` (int64) each
    rank's first global column.  torch.argmax returns the first maximum, i.e. the lowest rank
    among equal values.  Returns a 0-dim int64 tensor."""
    import torch

    pairs = slots.view(-1, 2)
    vals = pairs[:, 1].contiguous().view(torch.float32)
    best = torch.argmax(vals)
    idx = pairs[:, 0].to(torch.int64) + offsets
    return torch.where(vals[best] > -1e30, idx[best], torch.zeros_like(idx[best]))


def distributed_argmax(local_pair, n: int, group=None) -> int:
    """All-gather each rank's 8-byte (index, value) argmax of its lm_head shard (instead of its
    logits: 8 bytes per rank rather than 4 * n / world) and combine them.  `local_pair` is a
    2-element int32 tensor as mgpu_argmax writes it (index, fp32 value bits)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    slots = torch.empty(2 * world, dtype=torch.int32, device=local_pair.device)
    dist.all_gather_into_tensor(slots, local_pair.to(torch.int32).contiguous(), group=group)
    s = slots.cpu()
    vals = s.view(torch.float32)
    pairs = [(int(s[2 * r]), float(vals[2 * r + 1])) for r in range(world)]
    return combine_argmax(pairs, n, world)

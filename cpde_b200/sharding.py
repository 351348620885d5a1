"""Point-sharded engine groups: one process per GPU, one engine per process.

Every sample of a cPDE epoch is independent until the point-axis sums (loss,
weight gradients), so a group of engines splits each Data object's samples
into contiguous shards and sums gradients and cost totals over the group with
NCCL once per epoch. Every rank issues the same requests in the same order;
the engines slice what they keep.

    from cpde_b200 import sharding
    engine = sharding.engine(local_rank)      # inside torch.distributed ranks
"""
from . import native


def shard_range(total, rank, world):
    """(first sample, sample count) of ``rank``'s contiguous shard; the
    remainder ``total % world`` goes one sample each to the first ranks. Same
    rule as ``cpde_shard_range`` in the C ABI."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError('invalid shard request')
    base, extra = divmod(total, world)
    return rank * base + min(rank, extra), base + (1 if rank < extra else 0)


def exchange_id(make_id=native.sharding_id, group=None):
    """Rank 0 creates the NCCL group id with ``make_id`` and every rank of the
    torch.distributed ``group`` receives it (any backend, gloo included)."""
    import torch.distributed as dist
    payload = [make_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(payload, src=0, group=group)
    return payload[0]


def engine(device, group=None):
    """This rank's engine of a group spanning the torch.distributed ``group``
    (a single-device engine when the group has one rank)."""
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return native.Engine(device)
    uid = exchange_id(group=group)
    return native.Engine(device, dist.get_rank(group), dist.get_world_size(group), uid)

"""Edge sharding over the GPUs of one node (one process per GPU).

Edges are independent, so the path shards with no data-path collective: rank r
owns a contiguous, near-equal range of the edge list and writes its outputs
locally.  The only exchange is the replication of keyframe feature maps, one
NCCL broadcast from rank 0 (the reference runs on one GPU and has no
counterpart; cuda_slam/main.cu:1555-1613 processes every edge itself).
"""
from __future__ import annotations

from typing import Tuple


def edge_range(num_edges: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, stop) of rank's contiguous share; shares differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(num_edges, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def replicate_frames(fmaps, src: int = 0, group=None) -> None:
    """Broadcast keyframe feature maps [K, C, h, w] from rank `src` in place."""
    import torch.distributed as dist

    dist.broadcast(fmaps, src=src, group=group)


def replicate_store(dc, first_slot: int, count: int, src: int = 0, group=None) -> None:
    """Broadcast packed store slots from rank `src` (after its set_frames), so the
    other ranks skip packing: the packed fp16 pyramid is smaller than the fp32
    maps and identical on every rank."""
    import torch.distributed as dist

    dist.broadcast(dc.store_slots(first_slot, count), src=src, group=group)

"""Edge sharding over the GPUs of one node (one process per GPU).

Edges are independent, so the path shards with no data-path collective: rank r
owns a contiguous, near-equal range of the edge list and writes its outputs
locally.  The only exchange is the replication of keyframes, one NCCL
broadcast from rank 0: either of the raw feature maps (`replicate_frames`) or of
the packed store slots (`replicate_store`).  The reference runs on one GPU and
has no counterpart (cuda_slam/main.cu:1555-1613 processes every edge itself).

Failure detection is on the host, between steps: every rank posts a heartbeat
for the step to the rendezvous store before it launches the step's collective,
and `peers_alive` tells the others, within a deadline, which ranks did not, so
that no rank enters a broadcast a dead peer will never join.  A collective that
is entered anyway ends with an error after `timeout_s` (`replicate_frames`).
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


def replicate_frames(fmaps, src: int = 0, group=None, timeout_s: float = None) -> None:
    """Broadcast keyframe feature maps [K, C, h, w] from rank `src` in place.
    With `timeout_s`, a peer that never joins makes this raise RuntimeError after
    that many seconds instead of blocking."""
    import datetime

    import torch.distributed as dist

    if timeout_s is None:
        dist.broadcast(fmaps, src=src, group=group)
        return
    work = dist.broadcast(fmaps, src=src, group=group, async_op=True)
    work.wait(timeout=datetime.timedelta(seconds=timeout_s))


def peers_alive(store, step: int, world: int, rank: int, timeout_s: float = 1.0):
    """Post this rank's heartbeat for `step` and wait up to `timeout_s` for the
    other ranks' heartbeats.  Returns the sorted list of ranks that did not post
    (empty when all are alive).  `store` is the rendezvous store
    (torch.distributed TCPStore / FileStore)."""
    import time

    store.set(f"dc_alive/{step}/{rank}", "1")
    keys = {r: f"dc_alive/{step}/{r}" for r in range(world) if r != rank}
    deadline = time.monotonic() + timeout_s
    missing = sorted(keys)
    while missing:
        missing = [r for r in missing if not store.check([keys[r]])]
        if not missing or time.monotonic() >= deadline:
            break
        time.sleep(0.01)
    return missing


def replicate_store(dc, first_slot: int, count: int, src: int = 0, group=None,
                    timeout_s: float = None) -> None:
    """Broadcast packed store slots from rank `src` (after its set_frames), so the
    other ranks skip packing: the packed fp16 pyramid is smaller than the fp32
    maps and identical on every rank.  The collective runs on the current CUDA
    stream.  With `timeout_s`, a peer that never joins makes this raise
    RuntimeError after that many seconds instead of blocking (pair it with
    `peers_alive` between steps, so that a dead peer is noticed before the
    collective is entered)."""
    import datetime

    import torch.distributed as dist

    buf = dc.store_slots(first_slot, count)
    if timeout_s is None:
        dist.broadcast(buf, src=src, group=group)
        return
    work = dist.broadcast(buf, src=src, group=group, async_op=True)
    work.wait(timeout=datetime.timedelta(seconds=timeout_s))


class SlotRing:
    """Keyframe slots of the packed store with spare slots, so that the next
    keyframes can be packed (and replicated) while kernels of earlier steps
    still read the old ones.

    The store holds `frames + spares` slots.  Logical keyframe f lives in
    physical slot `phys[f]`; the spare slots wait in a FIFO.  `begin(f)` names
    the slot that receives f's new feature map (the oldest spare); `commit(f)`
    makes it f's slot and queues f's old slot as a spare.  A slot handed out by
    begin() at step j was last read by kernels of step j - spares - 1, so the
    keyframe of step j may be prepared during step j - spares + 1.  Edge lists
    are given in logical ids and translated with `slots(ii)`.  (The reference
    stores keyframe k in DroidState::fmaps[k], cuda_slam/main.cu:755,
    synchronously, on one GPU.)"""

    def __init__(self, frames: int, spares: int = 1):
        self.phys = list(range(frames))
        self.spares = list(range(frames, frames + spares))

    @property
    def spare(self) -> int:
        return self.spares[0]

    def begin(self, f: int) -> int:
        return self.spares[0]

    def commit(self, f: int) -> None:
        new = self.spares.pop(0)
        self.spares.append(self.phys[f])
        self.phys[f] = new

    def slots(self, ids):
        return [self.phys[int(i)] for i in ids]

"""CPU tests of the multi-GPU host logic: edge partitioning and feature-map
replication, the latter with world_size-2 gloo process groups."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from slam_hands_b200 import configs
from slam_hands_b200.shard import edge_range


@pytest.mark.parametrize("E,W", [(2048, 8), (2048, 3), (48, 5), (0, 4), (3, 8)])
def test_edge_ranges_partition(E, W):
    seen = []
    for r in range(W):
        a, b = edge_range(E, W, r)
        seen.extend(range(a, b))
        assert b - a in (E // W, E // W + 1)
    assert seen == list(range(E))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from slam_hands_b200.shard import replicate_frames
    wl = configs.WORKLOADS["C2"]
    fm = torch.from_numpy(configs.make_fmaps_np(wl, frames=3)) if rank == 0 else \
        torch.zeros(3, wl.channels, wl.h, wl.w)
    replicate_frames(fm)
    ii, jj = configs.make_edges(configs.WORKLOADS["C5"])
    a, b = edge_range(len(ii), world, rank)
    q.put((rank, float(fm.double().sum()), a, b))
    dist.barrier()
    dist.destroy_process_group()


def test_replication_and_sharding_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = float(torch.from_numpy(configs.make_fmaps_np(configs.WORKLOADS["C2"], frames=3)).double().sum())
    assert all(abs(r[1] - ref) < 1e-6 * max(1.0, abs(ref)) for r in res)
    assert res[0][2] == 0 and res[0][3] == res[1][2] and res[1][3] == 2048


def _failing_worker(rank, world, port, q):
    # rank 1 fails before step 1 (raises on the host, joins nothing); rank 0
    # learns of it from the missing heartbeat and skips the step's broadcast,
    # and a broadcast entered anyway ends with an error after its deadline
    from datetime import timedelta

    from slam_hands_b200.shard import peers_alive, replicate_frames, replicate_store

    class _Store:  # a context's packed slots, as a host tensor (gloo runs on CPU)
        def __init__(self):
            self.buf = torch.zeros(64, dtype=torch.uint8)

        def store_slots(self, first, count):
            return self.buf

    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))
    fm = torch.ones(2, 4, 3, 5) * (rank + 1)
    missing0 = peers_alive(store, 0, world, rank, timeout_s=10.0)
    replicate_frames(fm)  # step 0: everyone alive
    if rank == 1:
        q.put((rank, missing0, None, None))
        store.set("dc_test/rank1_done", "1")
        return  # "fails": no heartbeat for step 1, never joins again
    missing1 = peers_alive(store, 1, world, rank, timeout_s=1.0)
    store.wait(["dc_test/rank1_done"])
    raised = []
    for fn in (lambda: replicate_frames(fm, timeout_s=1.0),
               lambda: replicate_store(_Store(), 0, 1, timeout_s=1.0)):
        try:
            fn()
            raised.append(False)
        except RuntimeError:
            raised.append(True)
    q.put((rank, missing0, missing1, raised))
    q.close()
    q.join_thread()  # flush the result before the hard exit
    os._exit(0)  # the process group cannot be torn down with a dead peer


def test_dead_rank_detected_on_host_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict((r[0], r) for r in (q.get(timeout=120) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
    assert res[1][1] == [] and res[0][1] == []      # step 0: all heartbeats present
    assert res[0][2] == [1]                          # step 1: rank 1 reported missing
    assert res[0][3] == [True, True]                 # broadcasts entered anyway error out


def test_slot_ring_keeps_a_spare_slot():
    from slam_hands_b200.shard import SlotRing
    ring = SlotRing(4)
    assert ring.slots([0, 1, 2, 3]) == [0, 1, 2, 3] and ring.spare == 4
    for k in range(9):
        f = k % 4
        new = ring.begin(f)
        old = ring.phys[f]
        ring.commit(f)
        assert ring.phys[f] == new and ring.spare == old
        assert sorted(ring.phys + [ring.spare]) == list(range(5))  # a permutation of the slots


def test_slot_ring_with_two_spares_reuses_a_slot_three_steps_later():
    from slam_hands_b200.shard import SlotRing
    ring = SlotRing(3, spares=2)
    written = []
    for k in range(12):
        f = k % 3
        written.append(ring.begin(f))
        ring.commit(f)
        assert sorted(ring.phys + ring.spares) == list(range(5))
    # a slot handed out at step j held keyframe data read up to step j - 3
    for j in range(3, 12):
        assert written[j] not in written[j - 2:j]

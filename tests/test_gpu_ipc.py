"""Replication of packed keyframes between processes through CUDA IPC and the
copy engines (dc_store_ipc_handle / dc_store_attach_source /
dc_store_pull_slots) and the stream-ordered counters (dc_sync_signal /
dc_sync_wait): a second process on the same GPU opens the first one's store,
waits for the owner's counter, pulls slots, writes a counter back into the
owner's page, and its fused lookup is bit-identical to the owner's.  Every
counter wait is issued only after its value is known to be written."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

H, W, K, M = 24, 32, 4, 5


def _inputs():
    from slam_hands_b200 import configs
    rng = np.random.default_rng(3)
    fm = rng.standard_normal((K, 128, H, W), dtype=np.float32)
    ii = np.array([0, 1, 2, 3, 1], np.int32)
    jj = np.array([1, 2, 3, 0, 3], np.int32)
    coords = (configs.grid_coords(H, W)[None] + rng.normal(0, 2, (M, 2, H, W))).astype(np.float32)
    return fm, ii, jj, coords


def _puller(handle, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from slam_hands_b200 import DroidCorrelation
    try:
        fm, ii, jj, coords = _inputs()
        dc = DroidCorrelation(H, W, precision="fp16", max_frames=K)
        dc.attach_source(handle)
        # the owner set its counter before starting this process: satisfied at once
        dc.sync_wait(0, 5, remote=True)
        dc.pull_slots(0, K)
        dc.sync_signal(1, 7, remote=True)  # tell the owner, in its page
        out = dc.build_and_lookup(ii, jj, torch.from_numpy(coords).cuda())
        q.put(out.cpu().numpy())
        dc.close()
    except Exception as ex:  # report to the parent
        q.put(repr(ex))


def test_pull_slots_from_another_process(cuda):
    from slam_hands_b200 import DroidCorrelation
    fm, ii, jj, coords = _inputs()
    dc = DroidCorrelation(H, W, precision="fp16", max_frames=K)
    dc.set_frames(torch.from_numpy(fm).cuda())
    ref = dc.build_and_lookup(ii, jj, torch.from_numpy(coords).cuda()).cpu().numpy()
    dc.sync_signal(0, 5)
    torch.cuda.synchronize()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_puller, args=(dc.store_ipc_handle(), q))
    p.start()
    got = q.get(timeout=300)
    p.join(timeout=120)
    assert not isinstance(got, str), got
    assert p.exitcode == 0
    assert np.array_equal(got, ref)
    # the puller's remote write landed in this process's counter page (read
    # with a plain copy: no wait that could block)
    slots = dc.store_slots(0, K)
    base = slots.data_ptr() + slots.numel()

    class _Page:
        __cuda_array_interface__ = {"shape": (8,), "typestr": "<u4", "data": (base, False),
                                    "version": 3}

    page = torch.as_tensor(_Page(), device="cuda").cpu().tolist()
    assert page[0] == 5 and page[1] == 7

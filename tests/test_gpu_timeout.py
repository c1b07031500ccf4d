"""The fused kernel's bounded device-side waits, made to run out on purpose.

dc_debug_inject_stall(limit) makes every CTA withhold its first
source-tile load, so the MMA warp waits on a barrier that nothing will
complete.  After `limit` ns the wait gives up: the kernel raises the device
error word, every role leaves its loop, the copies in flight land, tensor
memory is freed and the kernel returns.  No fault, trap or unbounded wait is
involved.  The host then reads DC_ERR_DEVICE_TIMEOUT from dc_device_status,
and the same context computes exact results on the next call.
"""
import math

import numpy as np
import pytest
import torch

from slam_hands_b200 import _lib as L

from test_gpu_parity import normwise, oracle_alt, setup

pytestmark = pytest.mark.gpu

LIMIT_NS = 2_000_000  # 2 ms


@pytest.mark.parametrize("precision", ["fp16", "bf16"])
def test_wait_timeout_is_reported_and_context_survives(cuda, oracle, precision):
    lib = L.load()
    h, w = 48, 64
    alpha = 1 / math.sqrt(128)
    dc, fm, ii, jj, coords = setup(h, w, K=4, precision=precision, M=6, sigma=2.0, alpha=alpha)
    c = torch.from_numpy(coords).cuda()
    assert lib.dc_device_status(dc._ctx, None) == L.DC_OK
    try:
        assert lib.dc_debug_inject_stall(LIMIT_NS) == L.DC_OK
        dc.build_and_lookup(ii, jj, c)  # enqueues; the time-out is reported below
        st = lib.dc_device_status(dc._ctx, None)
    finally:
        lib.dc_debug_inject_stall(0)
    assert st == L.DC_ERR_DEVICE_TIMEOUT, st
    assert b"timed out" in lib.dc_last_error(dc._ctx)
    # the word was cleared by the read; the context computes exact results again
    assert lib.dc_device_status(dc._ctx, None) == L.DC_OK
    out = dc.build_and_lookup(ii, jj, c).cpu().numpy()
    assert lib.dc_device_status(dc._ctx, None) == L.DC_OK
    exp = oracle_alt(oracle, fm, ii, jj, coords, alpha, precision)
    assert normwise(out, exp) < 1e-4

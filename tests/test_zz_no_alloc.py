"""GPU test of dc_build_and_lookup_static, the entry point for callers that may
not allocate device memory (their memory belongs to another allocator or a
fixed arena): it must give the same output as dc_build_and_lookup, which packs
the keyframes into a context it allocated, on two calls in a row (the second
call finds the first call's data in the shared static array).  After every
call, dc_static_device_status must report no time-out; a time-out that the
test provokes on purpose (dc_debug_inject_stall: a barrier nothing completes,
a bounded wait that gives up) must be reported by it, and the next call must
be exact again.  The packed store's 32 MiB limit: the largest store that fits
(18 fp16 keyframes at 54x96x128) is accepted and exact, one frame more is
refused.

This file is collected last (test_zz_*), so a run that stops at the first
failure has run every other test before it."""
import ctypes
import math

import numpy as np
import pytest
import torch

from slam_hands_b200 import DroidCorrelation, configs
from slam_hands_b200 import _lib as L

pytestmark = pytest.mark.gpu

TOL = 1e-5  # normwise, the fp32 bar of the parity tests (both paths run the same kernels)
SCRATCH_BYTES = 32 << 20


def _case(seed, h, w, K, M, sigma):
    rng = np.random.default_rng(seed)
    fm = rng.standard_normal((K, 128, h, w), dtype=np.float32)
    ii = rng.integers(0, K, M).astype(np.int32)
    jj = ((ii + 1 + rng.integers(0, K - 1, M)) % K).astype(np.int32)
    coords = (configs.grid_coords(h, w)[None] + rng.normal(0, sigma, (M, 2, h, w))).astype(np.float32)
    return fm, ii, jj, coords


def _static_call(lib, cfg, fmt, K, ii_d, jj_d, M, c_d, out):
    return lib.dc_build_and_lookup_static(ctypes.byref(cfg), fmt.data_ptr(), L.DC_DTYPE_F32, K,
                                          ii_d.data_ptr(), jj_d.data_ptr(), M, c_d.data_ptr(),
                                          out.data_ptr(), torch.cuda.current_stream().cuda_stream)


def _config(lib, h, w, precision, alpha):
    cfg = L.DcConfig()
    lib.dc_default_config(ctypes.byref(cfg), h, w)
    cfg.precision = L.PRECISIONS[precision]
    cfg.alpha = alpha
    return cfg


def _run_pair(lib, precision, seed, h, w, K, M, sigma):
    """(context-path output, static-path output, static status) for one case."""
    alpha = 1 / math.sqrt(128)
    fm, ii, jj, coords = _case(seed, h, w, K, M, sigma)
    dc = DroidCorrelation(h, w, precision=precision, alpha=alpha, max_frames=K, max_edges=M)
    fmt = torch.from_numpy(fm).cuda()
    dc.set_frames(fmt)
    ii_d = torch.from_numpy(ii).cuda()
    jj_d = torch.from_numpy(jj).cuda()
    c_d = torch.from_numpy(coords).cuda()
    ref = dc.build_and_lookup(ii_d, jj_d, c_d).cpu().numpy()
    dc.close()
    out = torch.full((M, 196, h, w), float("nan"), device="cuda")
    rc = _static_call(lib, _config(lib, h, w, precision, alpha), fmt, K, ii_d, jj_d, M, c_d, out)
    assert rc == L.DC_OK, f"status {rc}"
    st = lib.dc_static_device_status(None)
    return ref, out.cpu().numpy(), st


def _normwise(got, ref):
    return float(np.abs(got - ref).max() / np.abs(ref).max())


@pytest.mark.parametrize("precision", ["fp16", "bf16", "fp32"])
def test_static_entry_matches_context_entry_twice(cuda, precision):
    lib = L.load()
    for call, case in enumerate([(1, 48, 64, 6, 7, 2.0), (2, 41, 73, 4, 5, 6.0)]):
        ref, got, st = _run_pair(lib, precision, *case)
        assert st == L.DC_OK, f"call {call}: device status {st}"
        err = _normwise(got, ref)
        assert np.isfinite(got).all() and err <= TOL, f"call {call}: normwise {err:.3e}"


def test_static_entry_largest_store_and_one_frame_more(cuda):
    lib = L.load()
    h, w = 54, 96
    rows = sum(-(-((h >> l) * (w >> l)) // 128) * 128 for l in range(4))
    K = SCRATCH_BYTES // (rows * 128 * 2)
    assert K == 18
    ref, got, st = _run_pair(lib, "fp16", 3, h, w, K, 4, 3.0)
    assert st == L.DC_OK
    assert _normwise(got, ref) <= TOL
    cfg = _config(lib, h, w, "fp16", 1 / 16)
    dummy = torch.zeros(1, device="cuda")
    e = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.dc_build_and_lookup_static(ctypes.byref(cfg), dummy.data_ptr(), L.DC_DTYPE_F32,
                                        K + 1, e.data_ptr(), e.data_ptr(), 1, dummy.data_ptr(),
                                        dummy.data_ptr(), None)
    assert rc == L.DC_ERR_INVALID_ARG


def test_static_entry_reports_a_timeout(cuda):
    lib = L.load()
    h, w, K, M = 48, 64, 4, 5
    fm, ii, jj, coords = _case(4, h, w, K, M, 2.0)
    fmt = torch.from_numpy(fm).cuda()
    ii_d = torch.from_numpy(ii).cuda()
    jj_d = torch.from_numpy(jj).cuda()
    c_d = torch.from_numpy(coords).cuda()
    out = torch.zeros(M, 196, h, w, device="cuda")
    cfg = _config(lib, h, w, "fp16", 1 / 16)
    assert lib.dc_static_device_status(None) == L.DC_OK
    try:
        assert lib.dc_debug_inject_stall(2_000_000) == L.DC_OK
        assert _static_call(lib, cfg, fmt, K, ii_d, jj_d, M, c_d, out) == L.DC_OK
        st = lib.dc_static_device_status(None)
    finally:
        lib.dc_debug_inject_stall(0)
    assert st == L.DC_ERR_DEVICE_TIMEOUT
    assert lib.dc_static_device_status(None) == L.DC_OK  # cleared by the read
    assert _static_call(lib, cfg, fmt, K, ii_d, jj_d, M, c_d, out) == L.DC_OK
    assert lib.dc_static_device_status(None) == L.DC_OK
    dc = DroidCorrelation(h, w, precision="fp16", alpha=1 / 16, max_frames=K, max_edges=M)
    dc.set_frames(fmt)
    ref = dc.build_and_lookup(ii_d, jj_d, c_d).cpu().numpy()
    assert _normwise(out.cpu().numpy(), ref) <= TOL

"""GPU test of dc_build_and_lookup_static, the entry point for callers that may
not allocate device memory (their memory belongs to another allocator or a
fixed arena): it must give the same output as dc_build_and_lookup, which packs
the keyframes into a context it allocated, on two calls in a row (the second
call finds the first call's data in the shared static array)."""
import ctypes
import math

import numpy as np
import pytest
import torch

from slam_hands_b200 import DroidCorrelation, configs
from slam_hands_b200 import _lib as L

pytestmark = pytest.mark.gpu

TOL = 1e-5  # normwise, the fp32 bar of the parity tests (both paths run the same kernels)


def _case(seed, h, w, K, M, sigma):
    rng = np.random.default_rng(seed)
    fm = rng.standard_normal((K, 128, h, w), dtype=np.float32)
    ii = rng.integers(0, K, M).astype(np.int32)
    jj = ((ii + 1 + rng.integers(0, K - 1, M)) % K).astype(np.int32)
    coords = (configs.grid_coords(h, w)[None] + rng.normal(0, sigma, (M, 2, h, w))).astype(np.float32)
    return fm, ii, jj, coords


@pytest.mark.parametrize("precision", ["fp16", "fp32"])
def test_static_entry_matches_context_entry_twice(cuda, precision):
    lib = L.load()
    alpha = 1 / math.sqrt(128)
    for call, (seed, h, w, K, M, sigma) in enumerate([(1, 48, 64, 6, 7, 2.0), (2, 41, 73, 4, 5, 6.0)]):
        fm, ii, jj, coords = _case(seed, h, w, K, M, sigma)
        dc = DroidCorrelation(h, w, precision=precision, alpha=alpha, max_frames=K, max_edges=M)
        fmt = torch.from_numpy(fm).cuda()
        dc.set_frames(fmt)
        ii_d = torch.from_numpy(ii).cuda()
        jj_d = torch.from_numpy(jj).cuda()
        c_d = torch.from_numpy(coords).cuda()
        ref = dc.build_and_lookup(ii_d, jj_d, c_d).cpu().numpy()
        cfg = L.DcConfig()
        lib.dc_default_config(ctypes.byref(cfg), h, w)
        cfg.precision = L.PRECISIONS[precision]
        cfg.alpha = alpha
        out = torch.full((M, 196, h, w), float("nan"), device="cuda")
        rc = lib.dc_build_and_lookup_static(ctypes.byref(cfg), fmt.data_ptr(), L.DC_DTYPE_F32, K,
                                            ii_d.data_ptr(), jj_d.data_ptr(), M, c_d.data_ptr(),
                                            out.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert rc == L.DC_OK, f"call {call}: status {rc}"
        got = out.cpu().numpy()
        err = float(np.abs(got - ref).max() / np.abs(ref).max())
        assert np.isfinite(got).all() and err <= TOL, f"call {call}: normwise {err:.3e}"
        dc.close()


def test_static_entry_rejects_oversized_store(cuda):
    lib = L.load()
    cfg = L.DcConfig()
    lib.dc_default_config(ctypes.byref(cfg), 54, 96)
    dummy = torch.zeros(1, device="cuda")
    e = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.dc_build_and_lookup_static(ctypes.byref(cfg), dummy.data_ptr(), L.DC_DTYPE_F32, 1000,
                                        e.data_ptr(), e.data_ptr(), 1, dummy.data_ptr(),
                                        dummy.data_ptr(), None)
    assert rc == L.DC_ERR_INVALID_ARG

"""CPU tests pinning the oracle to the reference's own kernels.

tests/golden/reference_kernels.npz holds seeded inputs and the outputs of the
reference kernels (cuda_slam/main.cu:1077-1217 rebuilt for sm_100a, cuBLAS FP16
for the volume) produced on a B200 by tests/golden/make_golden.py.  The oracle
must reproduce the lookup and pooling outputs bit for bit, and the whole FP16
pipeline within the FP16-mode tolerance (cuBLAS sums in its own order).
"""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_kernels.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


def test_oracle_lookup_batched_bit_exact(oracle, gold):
    vols = [gold[f"lookup_vol{l}"] for l in range(4)]
    h, w = vols[1].shape[-2] * 2, vols[1].shape[-1] * 2
    out = oracle.lookup(vols, gold["lookup_coords"], h, w, 3, oracle.LOOKUP_BATCHED)
    assert np.array_equal(out, gold["lookup_batched_out"])


def test_oracle_lookup_single_bit_exact(oracle, gold):
    vols = [gold[f"lookup_vol{l}"][:1] for l in range(4)]
    h, w = vols[1].shape[-2] * 2, vols[1].shape[-1] * 2
    out = oracle.lookup(vols, gold["lookup_coords"][:1], h, w, 3, oracle.LOOKUP_SINGLE)[0]
    assert np.array_equal(out, gold["lookup_single_out"])


def test_oracle_pool_bit_exact(oracle, gold):
    assert np.array_equal(oracle.pool2x2(gold["pool_in"]), gold["pool_out"])


def test_oracle_pipeline_fp16(oracle, gold):
    fm = gold["pipe_fmaps"]
    ii, jj, coords = gold["pipe_ii"], gold["pipe_jj"], gold["pipe_coords"]
    alpha = float(gold["pipe_alpha"])
    h, w = fm.shape[-2:]
    fm16 = fm.astype(np.float16).astype(np.float32)  # DroidState::fmaps is __half
    for e in range(len(ii)):
        V = oracle.volume_f64(fm16[ii[e]], fm16[jj[e]], alpha)
        ref_v = gold["pipe_vol0"][e]
        assert np.abs(V - ref_v).max() / np.abs(ref_v).max() < 1e-5
        out = oracle.lookup(oracle.pyramid(V[None], h, w, 4), coords[e:e + 1], h, w, 3)[0]
        ref = gold["pipe_out"][e]
        assert np.abs(out - ref).max() / np.abs(ref).max() < 1e-5

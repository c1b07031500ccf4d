"""GraphAgg scatter-mean (dc_scatter_mean, main.cu:2255-2294) and the update
step's per-edge row gather (dc_gather_rows, main.cu:2215-2224).

CPU: the oracle (orc_scatter_mean, the reference's memset + per-edge
scale_add_kernel + per-keyframe scale loop) against plain numpy means.
GPU: the library's one-kernel version against the oracle, bit for bit."""
import numpy as np
import pytest
import torch

from slam_hands_b200 import DroidCorrError, DroidCorrelation


def test_oracle_is_the_mean_in_ascending_keyframe_order(oracle):
    rng = np.random.default_rng(0)
    feats = rng.standard_normal((9, 4, 5, 6), dtype=np.float32)
    ii = np.array([4, 1, 4, 9, 1, 4, 2, 9, 4], np.int32)
    agg, ids = oracle.scatter_mean(feats, ii)
    assert list(ids) == [1, 2, 4, 9]
    for k, kf in enumerate(ids):
        exp = feats[ii == kf].astype(np.float64).mean(0)
        assert np.abs(agg[k] - exp).max() < 1e-6
    assert np.array_equal(agg[1], feats[6])  # one edge: copied exactly


@pytest.mark.gpu
@pytest.mark.parametrize("E,shape", [(48, (128, 48, 64)), (13, (3, 7, 9)), (1, (128, 12, 16))])
def test_scatter_mean_bit_exact_vs_oracle(cuda, oracle, E, shape):
    rng = np.random.default_rng(E)
    feats = rng.standard_normal((E,) + shape, dtype=np.float32)
    ii = rng.integers(0, max(2, E // 3), E).astype(np.int32)
    dc = DroidCorrelation(12, 16, max_frames=4, max_edges=64)
    agg, ids = dc.scatter_mean(torch.from_numpy(feats).cuda(), ii)
    exp, exp_ids = oracle.scatter_mean(feats, ii)
    assert np.array_equal(ids, exp_ids)
    assert np.array_equal(agg.cpu().numpy(), exp)


@pytest.mark.gpu
def test_scatter_mean_rejects_too_many_edges(cuda):
    dc = DroidCorrelation(12, 16, max_frames=4, max_edges=4)
    with pytest.raises(DroidCorrError):
        dc.scatter_mean(torch.zeros(5, 8, device="cuda"), [0, 1, 2, 3, 0])


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(128, 48, 64), (5, 7, 3)])
def test_gather_rows_exact(cuda, shape):
    # the update step's per-edge inps[ii[e]] loads (main.cu:2215-2224) in one launch
    rng = np.random.default_rng(7)
    src = rng.standard_normal((12,) + shape, dtype=np.float32)
    idx = np.array([3, 0, 11, 3, 7, -1, 12, 5], np.int32)  # two out of range
    dc = DroidCorrelation(12, 16, max_frames=4, max_edges=8)
    got = dc.gather_rows(torch.from_numpy(src).cuda(), idx).cpu().numpy()
    for e, r in enumerate(idx):
        exp = src[r] if 0 <= r < 12 else np.zeros(shape, np.float32)
        assert np.array_equal(got[e], exp)


@pytest.mark.gpu
@pytest.mark.parametrize("E,shape", [(48, (128, 48, 64)), (13, (3, 7, 9))])
def test_scatter_mean_bit_exact_vs_reference_kernel(cuda, E, shape):
    # the reference's own loop on the GPU: memset, scale_add_kernel per edge and
    # per keyframe (main.cu:2262-2294, nn.cuh:381-385), built into oracle/_ref
    from oracle import ref as REF
    if not REF.available():
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(100 + E)
    feats = rng.standard_normal((E,) + shape, dtype=np.float32)
    ii = rng.integers(0, max(2, E // 3), E).astype(np.int32)
    dc = DroidCorrelation(12, 16, max_frames=4, max_edges=64)
    agg, ids = dc.scatter_mean(torch.from_numpy(feats).cuda(), ii)
    ref, ref_ids = REF.scatter_mean(feats, ii)
    assert np.array_equal(ids, ref_ids)
    assert np.array_equal(agg.cpu().numpy(), ref)

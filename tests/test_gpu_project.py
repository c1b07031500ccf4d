"""GPU parity of the reprojection (dc_project) and of the projection + fused
correlation entry point (dc_project_build_and_lookup).

Bars:
  - coordinates: max |our - oracle| <= 2e-3 px against the float64 oracle
    (oracle.project, a restatement of cuda_slam/se3.cuh:118-177) and against the
    reference's own projmap_kernel + batch_coords_hw2_to_2hw run on the GPU
    (the reference is built with --use_fast_math, so agreement is to a few
    float ulps of coordinates up to ~100 px, not bit for bit);
  - valid mask: equal wherever the projected depth is not within 1e-4 of the
    0.25 threshold;
  - dc_project_build_and_lookup: bit-identical to dc_project followed by
    dc_build_and_lookup on the same coordinates (same kernels, same inputs).
"""
import math

import numpy as np
import pytest
import torch

from oracle import ref as REF
from slam_hands_b200 import DroidCorrelation, configs

pytestmark = pytest.mark.gpu

TOL_PX = 2e-3
needs_ref = pytest.mark.skipif(not REF.available(), reason="oracle/_ref not built")


def scene(h, w, N, seed):
    rng = np.random.default_rng(seed)
    poses = configs.random_poses(N, rng, trans=0.15, angle=0.08)
    disps = rng.uniform(0.15, 1.2, (N, h, w)).astype(np.float32)
    intr = np.array([0.95 * w, 0.95 * w, w / 2 - 0.5, h / 2 - 0.5], np.float32)
    return poses, disps, intr


def depth_near_threshold(poses, disps, intr, ii, jj):
    # projected depth z * d of every pixel, to exclude ties at MIN_DEPTH
    from oracle import oracle as O
    N, H, W = disps.shape
    v, u = np.meshgrid(np.arange(H, dtype=np.float64), np.arange(W, dtype=np.float64),
                       indexing="ij")
    near = []
    for i, j in zip(ii, jj):
        if not (0 <= i < N and 0 <= j < N):
            near.append(np.zeros((H, W), bool))
            continue
        tij, qij = O.relative_pose(poses[i].astype(np.float64), poses[j].astype(np.float64))
        Xi = np.stack([(u - intr[2]) / intr[0], (v - intr[3]) / intr[1], np.ones_like(u)], -1)
        z = O._rotate(qij, Xi)[..., 2] + disps[i] * tij[2]
        near.append(np.abs(z - 0.25) < 1e-4)
    return np.array(near)


@pytest.mark.parametrize("h,w", [(48, 64), (41, 73)])
def test_project_vs_oracle(cuda, oracle, h, w):
    N = 6
    poses, disps, intr = scene(h, w, N, seed=h)
    ii = np.array([0, 1, 2, 3, 4, 5, 0, 3], np.int32)
    jj = np.array([1, 2, 3, 4, 5, 0, 5, 1], np.int32)
    dc = DroidCorrelation(h, w, precision="fp16", max_frames=N, max_edges=len(ii))
    coords, valid = dc.project(torch.from_numpy(poses).cuda(), torch.from_numpy(disps).cuda(),
                               torch.from_numpy(intr).cuda(), ii, jj)
    exp_c, exp_v = oracle.project(poses, disps, intr, ii, jj)
    err = float(np.abs(coords.cpu().numpy() - exp_c).max())
    print(f"project {h}x{w}: max |coords - oracle| = {err:.2e} px")
    assert err < TOL_PX
    near = depth_near_threshold(poses, disps, intr, ii, jj)
    got_v = valid.cpu().numpy()
    assert np.array_equal(got_v[~near], exp_v[~near])
    assert got_v.mean() > 0.9  # small motions: nearly every pixel lands in front


@needs_ref
def test_project_vs_reference_kernel(cuda):
    h, w, N = 48, 64, 8
    poses, disps, intr = scene(h, w, N, seed=5)
    ii = np.array([0, 1, 2, 3, 4, 5, 6, 7, 2, 5], np.int32)
    jj = np.array([1, 2, 3, 4, 5, 6, 7, 0, 6, 1], np.int32)
    ref_c, ref_v = REF.project(poses, disps, intr, ii, jj)
    dc = DroidCorrelation(h, w, precision="fp16", max_frames=N, max_edges=len(ii))
    coords, valid = dc.project(torch.from_numpy(poses).cuda(), torch.from_numpy(disps).cuda(),
                               torch.from_numpy(intr).cuda(), ii, jj)
    err = float(np.abs(coords.cpu().numpy() - ref_c).max())
    print(f"project vs reference projmap_kernel: max |coords diff| = {err:.2e} px")
    assert err < TOL_PX
    near = depth_near_threshold(poses, disps, intr, ii, jj)
    assert np.array_equal(valid.cpu().numpy()[~near], ref_v[~near])


def test_project_invalid_edges_and_behind_camera(cuda, oracle):
    h, w, N = 12, 16, 2
    poses = np.zeros((N, 7), np.float32)
    poses[:, 6] = 1.0
    poses[1, 2] = -5.0  # everything lands behind frame 1's camera
    disps = np.ones((N, h, w), np.float32)
    intr = np.array([10.0, 10.0, 7.5, 5.5], np.float32)
    ii = np.array([0, 0, -1], np.int32)
    jj = np.array([1, 9, 0], np.int32)
    dc = DroidCorrelation(h, w, precision="fp32", max_frames=N, max_edges=3)
    coords, valid = dc.project(torch.from_numpy(poses).cuda(), torch.from_numpy(disps).cuda(),
                               torch.from_numpy(intr).cuda(), ii, jj)
    grid = configs.grid_coords(h, w)
    for e in range(3):
        assert np.array_equal(coords[e].cpu().numpy(), grid)
    assert np.all(valid.cpu().numpy() == 0.0)


@pytest.mark.parametrize("precision", ["fp16", "fp32"])
def test_project_build_and_lookup_equals_two_calls(cuda, precision):
    h, w, N = 48, 64, 6
    poses, disps, intr = scene(h, w, N, seed=11)
    rng = np.random.default_rng(3)
    fm = torch.from_numpy(rng.standard_normal((N, 128, h, w), dtype=np.float32)).cuda()
    ii = np.array([0, 1, 2, 3, 4, 5, 1, 4], np.int32)
    jj = np.array([1, 2, 3, 4, 5, 0, 3, 0], np.int32)
    dc = DroidCorrelation(h, w, precision=precision, alpha=1 / math.sqrt(128), max_frames=N,
                          max_edges=len(ii))
    dc.set_frames(fm)
    P, Dp, I = (torch.from_numpy(a).cuda() for a in (poses, disps, intr))
    out, coords, valid = dc.project_build_and_lookup(P, Dp, I, ii, jj)
    c2, v2 = dc.project(P, Dp, I, ii, jj)
    out2 = dc.build_and_lookup(ii, jj, c2)
    assert dc.lib.dc_device_status(dc._ctx, None) == 0
    assert torch.equal(coords, c2) and torch.equal(valid, v2)
    assert torch.equal(out, out2)
    assert torch.isfinite(out).all()

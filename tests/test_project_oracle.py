"""The reprojection oracle (oracle.project) against textbook rigid-body
geometry, on CPU: rotation-matrix form of the quaternion, camera-from-world
poses, pinhole projection.  Pins the conventions the reference uses
(cuda_slam/se3.cuh:8-55, :118-177) before the CUDA kernel is checked against it."""
import numpy as np

from oracle import oracle as O
from slam_hands_b200.configs import random_poses


def quat_to_R(q):
    x, y, z, w = q
    return np.array([
        [1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)],
        [2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)],
        [2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)]])


def test_identity_relative_pose_keeps_the_grid():
    rng = np.random.default_rng(0)
    poses = random_poses(3, rng)
    disps = rng.uniform(0.2, 2.0, (3, 6, 8))
    coords, valid = O.project(poses, disps, (50.0, 50.0, 4.0, 3.0), [1, 2], [1, 2])
    v, u = np.meshgrid(np.arange(6), np.arange(8), indexing="ij")
    assert np.allclose(coords[:, 0], u) and np.allclose(coords[:, 1], v)
    assert np.all(valid == 1.0)


def test_projection_matches_matrix_geometry():
    rng = np.random.default_rng(1)
    N, H, W = 4, 5, 7
    poses = random_poses(N, rng, trans=0.3, angle=0.2).astype(np.float64)
    poses[:, 3:] /= np.linalg.norm(poses[:, 3:], axis=1, keepdims=True)  # exactly unit in f64
    disps = rng.uniform(0.3, 1.5, (N, H, W))
    fx, fy, cx, cy = 60.0, 55.0, 3.2, 2.1
    ii, jj = [0, 2, 3], [1, 0, 2]
    coords, valid = O.project(poses, disps, (fx, fy, cx, cy), ii, jj)
    for e, (i, j) in enumerate(zip(ii, jj)):
        Ri, Rj = quat_to_R(poses[i, 3:]), quat_to_R(poses[j, 3:])
        for y in range(H):
            for x in range(W):
                d = disps[i, y, x]
                Pc = np.array([(x - cx) / fx, (y - cy) / fy, 1.0]) / d   # camera i point
                Pw = Ri.T @ (Pc - poses[i, :3])                          # world
                Q = Rj @ Pw + poses[j, :3]                               # camera j
                assert abs(coords[e, 0, y, x] - (fx * Q[0] / Q[2] + cx)) < 1e-9
                assert abs(coords[e, 1, y, x] - (fy * Q[1] / Q[2] + cy)) < 1e-9
                assert valid[e, y, x] == float(Q[2] * d > 0.25)


def test_behind_camera_and_invalid_edges_keep_the_pixel():
    poses = np.zeros((2, 7), np.float32)
    poses[:, 6] = 1.0
    poses[1, 2] = -5.0          # frame 1 is 5 units behind along z
    disps = np.ones((2, 3, 4), np.float32)
    coords, valid = O.project(poses, disps, (10.0, 10.0, 1.5, 1.0), [0, 0], [1, 7])
    v, u = np.meshgrid(np.arange(3), np.arange(4), indexing="ij")
    for e in range(2):
        assert np.array_equal(coords[e, 0], u) and np.array_equal(coords[e, 1], v)
        assert np.all(valid[e] == 0.0)

"""Generate the golden fixtures from the reference's own correlation kernels.

Runs on a GPU box: oracle/_ref/libref.so holds cuda_slam/main.cu:1077-1217
(corr_index_kernel, avg_pool_2x2_kernel, batch_corr_sample_kernel) compiled for
sm_100a and driven like CudaDroid (main.cu:1529-1613), with cuBLAS FP16 for the
volume build.  Inputs are seeded; inputs and reference outputs are saved
together in reference_kernels.npz so the CPU tests need no GPU and no reference
tree.

    python tests/golden/make_golden.py [output.npz]
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import ref as REF  # noqa: E402
from slam_hands_b200 import configs  # noqa: E402


def main():
    rng = np.random.default_rng(20261201)
    h, w = 12, 16
    hw = h * w
    out = {}
    # (a) batched lookup (batch_corr_sample_kernel x4) on random volumes,
    #     coordinates with negative fractions, integers and far out-of-bounds
    M = 2
    vols = [rng.standard_normal((M, hw, h >> l, w >> l), dtype=np.float32) for l in range(4)]
    coords = (configs.grid_coords(h, w)[None] + rng.uniform(-6, 6, (M, 2, h, w))).astype(np.float32)
    coords[:, :, 0, :3] = -0.5
    coords[:, :, 1, :3] = 3.0
    coords[:, :, 2, :3] = -1000.0
    for l in range(4):
        out[f"lookup_vol{l}"] = vols[l]
    out["lookup_coords"] = coords
    out["lookup_batched_out"] = REF.lookup_batched(vols, coords, h, w)
    # (b) single-edge lookup (corr_index_kernel x4)
    out["lookup_single_out"] = REF.lookup_single([v[0] for v in vols], coords[0], h, w)
    # (c) pooling on an odd grid (floor)
    x = rng.standard_normal((5, 41, 73), dtype=np.float32)
    out["pool_in"] = x
    out["pool_out"] = REF.pool(x)
    # (d) whole FP16 pipeline: fp16 fmaps, cublasGemmBatchedEx, pools, lookups
    fm = rng.standard_normal((3, 128, h, w), dtype=np.float32)
    ii = np.array([0, 2, 1], np.int32)
    jj = np.array([1, 0, 2], np.int32)
    c2 = (configs.grid_coords(h, w)[None] + rng.normal(0, 2, (3, 2, h, w))).astype(np.float32)
    alpha = 1.0 / 16.0
    res, vol0, _ = REF.build_and_sample_fp16(fm, ii, jj, c2, alpha, want_vol0=True)
    out.update(pipe_fmaps=fm, pipe_ii=ii, pipe_jj=jj, pipe_coords=c2,
               pipe_alpha=np.float32(alpha), pipe_out=res, pipe_vol0=vol0)
    dst = sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "reference_kernels.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst)


if __name__ == "__main__":
    main()

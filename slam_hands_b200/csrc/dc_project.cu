// dc_project.cu -- reprojection of source pixels into the target frame, written
// straight in the lookup's coordinate layout.
//
// Replaces the first two launches of the reference's per-batch update step
// (cuda_slam/main.cu:2188-2197): projmap_kernel (cuda_slam/se3.cuh:118-177)
// writing interleaved coords [M][H][W][2] plus a valid mask, followed by
// batch_coords_hw2_to_2hw (main.cu:1135-1146) converting them to [M][2][H][W]
// for the correlation lookup.  Here one kernel writes coords_2hw[e][0][p] = x,
// coords_2hw[e][1][p] = y and valid[e][p] directly (coalesced over p), so the
// interleaved buffer and the layout pass disappear;
// dc_project_build_and_lookup then runs the correlation on those coordinates.
//
// The geometry is the reference's (DROID-SLAM's SE3 conventions):
//   pose = (t_x, t_y, t_z, q_x, q_y, q_z, q_w) per frame, world -> camera;
//   relative pose G_ij = G_j * G_i^-1 (q_ij = q_j * conj(q_i),
//   t_ij = t_j - R(q_ij) t_i), se3.cuh:44-55;
//   homogeneous point X_i = ((u - cx) / fx, (v - cy) / fy, 1, d) with d the
//   inverse depth of frame ii at pixel (u, v); X_j = (R X_i[0:3] + d t, d)
//   (actSE3, se3.cuh:19-26, the rotation by the quaternion in the
//   "t = 2 q x v; v + w t + q x t" form of actSO3, se3.cuh:8-17);
//   coords = (fx X_j.x / X_j.z + cx, fy X_j.y / X_j.z + cy) when X_j.z > 0.01,
//   else the pixel itself; valid = X_j.z > 0.25 (MIN_DEPTH, se3.cuh:6).
// Every product and sum is written in the reference's order; the reference
// is compiled with --use_fast_math (approximate division), this library with
// IEEE division, so coordinates agree to a few float ulps, not bit for bit.
#include "dc_internal.cuh"

namespace {

constexpr float kZNear = 0.01f;    // below: keep the pixel's own coordinate
constexpr float kMinDepth = 0.25f; // above: valid

// v -> q v q*, for unit quaternion q = (x, y, z, w).
__device__ __forceinline__ void rotate(const float* q, const float* X, float* Y) {
    float uv[3];
    uv[0] = 2.0f * (q[1] * X[2] - q[2] * X[1]);
    uv[1] = 2.0f * (q[2] * X[0] - q[0] * X[2]);
    uv[2] = 2.0f * (q[0] * X[1] - q[1] * X[0]);
    Y[0] = X[0] + q[3] * uv[0] + (q[1] * uv[2] - q[2] * uv[1]);
    Y[1] = X[1] + q[3] * uv[1] + (q[2] * uv[0] - q[0] * uv[2]);
    Y[2] = X[2] + q[3] * uv[2] + (q[0] * uv[1] - q[1] * uv[0]);
}

// One thread per (edge, source pixel); every thread forms its edge's relative
// pose from the two frames' poses (a few dozen flops, uniform over the CTA).
__global__ void __launch_bounds__(256) project_kernel(
    const float* __restrict__ poses, const float* __restrict__ disps,
    const float* __restrict__ intrinsics, const int* __restrict__ ii,
    const int* __restrict__ jj, int num_frames, int H, int W, float* __restrict__ coords,
    float* __restrict__ valid) {
    const int e = blockIdx.y;
    const int hw = H * W;
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= hw) return;
    const int ix = __ldg(ii + e), jx = __ldg(jj + e);
    const int v_ = k / W, u_ = k - v_ * W;
    const float u = (float)u_, v = (float)v_;
    float* cx_out = coords + (size_t)e * 2 * hw + k;
    if (ix < 0 || ix >= num_frames || jx < 0 || jx >= num_frames) {
        cx_out[0] = u;  // no pose: the pixel stays where it is, and is not valid
        cx_out[hw] = v;
        if (valid) valid[(size_t)e * hw + k] = 0.0f;
        return;
    }
    const float fx = __ldg(intrinsics + 0), fy = __ldg(intrinsics + 1);
    const float cx = __ldg(intrinsics + 2), cy = __ldg(intrinsics + 3);
    float ti[3], tj[3], qi[4], qj[4];
#pragma unroll
    for (int c = 0; c < 3; c++) {
        ti[c] = __ldg(poses + ix * 7 + c);
        tj[c] = __ldg(poses + jx * 7 + c);
    }
#pragma unroll
    for (int c = 0; c < 4; c++) {
        qi[c] = __ldg(poses + ix * 7 + 3 + c);
        qj[c] = __ldg(poses + jx * 7 + 3 + c);
    }
    // G_ij = G_j G_i^-1
    float qij[4], tij[3];
    qij[0] = -qj[3] * qi[0] + qj[0] * qi[3] - qj[1] * qi[2] + qj[2] * qi[1];
    qij[1] = -qj[3] * qi[1] + qj[1] * qi[3] - qj[2] * qi[0] + qj[0] * qi[2];
    qij[2] = -qj[3] * qi[2] + qj[2] * qi[3] - qj[0] * qi[1] + qj[1] * qi[0];
    qij[3] = qj[3] * qi[3] + qj[0] * qi[0] + qj[1] * qi[1] + qj[2] * qi[2];
    rotate(qij, ti, tij);
    tij[0] = tj[0] - tij[0];
    tij[1] = tj[1] - tij[1];
    tij[2] = tj[2] - tij[2];

    const float d = __ldg(disps + (size_t)ix * hw + k);
    float Xi[3], Xj[3];
    Xi[0] = (u - cx) / fx;
    Xi[1] = (v - cy) / fy;
    Xi[2] = 1.0f;
    rotate(qij, Xi, Xj);
    Xj[0] += d * tij[0];
    Xj[1] += d * tij[1];
    Xj[2] += d * tij[2];
    if (Xj[2] > kZNear) {
        cx_out[0] = fx * (Xj[0] / Xj[2]) + cx;
        cx_out[hw] = fy * (Xj[1] / Xj[2]) + cy;
    } else {
        cx_out[0] = u;
        cx_out[hw] = v;
    }
    if (valid) valid[(size_t)e * hw + k] = Xj[2] > kMinDepth ? 1.0f : 0.0f;
}

}  // namespace

int dc_launch_project(dc_ctx* ctx, const float* poses, const float* disps,
                      const float* intrinsics, const int* ii, const int* jj, int M,
                      int num_frames, float* coords, float* valid, cudaStream_t s) {
    const int H = ctx->cfg.h, W = ctx->cfg.w;
    dim3 grid((H * W + 255) / 256, M);
    project_kernel<<<grid, 256, 0, s>>>(poses, disps, intrinsics, ii, jj, num_frames, H, W,
                                        coords, valid);
    return dc_check_launch(ctx, "project_kernel");
}

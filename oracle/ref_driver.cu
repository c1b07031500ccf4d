// ref_driver.cu -- host driver that runs the reference's own correlation kernels
// on a B200.  TEST INFRASTRUCTURE ONLY (the second checker, and the GPU timing of
// the reference); never part of the product path.
//
// The reference kernels are not committed here.  oracle/Makefile (target `ref`)
// extracts cuda_slam/main.cu:1077-1217 from the read-only reference tree into
// oracle/_ref/ref_kernels.cuh at build time; the whole main.cu cannot be compiled
// in this image (it needs FFmpeg headers, main.cu:26-30).  This file then
// reproduces the call sequence of the reference host methods:
//   CudaDroid::sample_correlation          cuda_slam/main.cu:1529-1552
//   CudaDroid::batch_build_and_sample_...  cuda_slam/main.cu:1555-1613
// built with the reference's flags (-O3 --use_fast_math, cuda_slam/Makefile:4)
// for sm_100a.  All entry points take HOST arrays and return 0 on success.
#include <cublas_v2.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <map>
#include <set>
#include <vector>

#include "ref_kernels.cuh"
#include "ref_nn.cuh"   // scale_add_kernel, nn.cuh:381-385
#include "se3.cuh"  // the reference header, included where it lies (-I cuda_slam)

#define RCHK(x)                                                                      \
    do {                                                                             \
        cudaError_t e_ = (x);                                                        \
        if (e_ != cudaSuccess) {                                                     \
            fprintf(stderr, "ref_driver: %s at %s:%d\n", cudaGetErrorString(e_),     \
                    __FILE__, __LINE__);                                             \
            return 2;                                                                \
        }                                                                            \
    } while (0)
#define BCHK(x)                                                                      \
    do {                                                                             \
        cublasStatus_t s_ = (x);                                                     \
        if (s_ != CUBLAS_STATUS_SUCCESS) {                                           \
            fprintf(stderr, "ref_driver: cublas %d at %s:%d\n", (int)s_, __FILE__,   \
                    __LINE__);                                                       \
            return 3;                                                                \
        }                                                                            \
    } while (0)

namespace {

__global__ void f32_to_f16(const float* in, __half* out, size_t n) {
    size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (i < n) out[i] = __float2half_rn(in[i]);
}

template <typename T>
struct DBuf {
    T* p = nullptr;
    ~DBuf() { if (p) cudaFree(p); }
    cudaError_t alloc(size_t n) { return cudaMalloc(&p, n * sizeof(T)); }
};

}  // namespace

extern "C" {

int ref_version(void) { return 3; }

// projmap_kernel (se3.cuh:118-177) then batch_coords_hw2_to_2hw
// (main.cu:1135-1146), as the update step launches them (main.cu:2188-2197).
// poses_h [N][7], disps_h [N][H][W], intr_h [4], ii_h / jj_h [M];
// coords_h [M][2][H][W], valid_h [M][H][W].
int ref_project(const float* poses_h, const float* disps_h, const float* intr_h, int N,
                const int* ii_h, const int* jj_h, int M, int H, int W, float* coords_h,
                float* valid_h) {
    const int hw = H * W;
    DBuf<float> poses, disps, intr, hw2, chw, valid;
    DBuf<int> ii, jj;
    RCHK(poses.alloc((size_t)N * 7));
    RCHK(disps.alloc((size_t)N * hw));
    RCHK(intr.alloc(4));
    RCHK(ii.alloc(M));
    RCHK(jj.alloc(M));
    RCHK(hw2.alloc((size_t)M * hw * 2));
    RCHK(chw.alloc((size_t)M * hw * 2));
    RCHK(valid.alloc((size_t)M * hw));
    RCHK(cudaMemcpy(poses.p, poses_h, (size_t)N * 7 * 4, cudaMemcpyHostToDevice));
    RCHK(cudaMemcpy(disps.p, disps_h, (size_t)N * hw * 4, cudaMemcpyHostToDevice));
    RCHK(cudaMemcpy(intr.p, intr_h, 16, cudaMemcpyHostToDevice));
    RCHK(cudaMemcpy(ii.p, ii_h, (size_t)M * 4, cudaMemcpyHostToDevice));
    RCHK(cudaMemcpy(jj.p, jj_h, (size_t)M * 4, cudaMemcpyHostToDevice));
    projmap_kernel<<<M, 256>>>(poses.p, disps.p, intr.p, ii.p, jj.p, hw2.p, valid.p, M, H, W);
    RCHK(cudaGetLastError());
    batch_coords_hw2_to_2hw<<<(M * hw + 255) / 256, 256>>>(hw2.p, chw.p, M, hw);
    RCHK(cudaGetLastError());
    RCHK(cudaMemcpy(coords_h, chw.p, (size_t)M * hw * 2 * 4, cudaMemcpyDeviceToHost));
    RCHK(cudaMemcpy(valid_h, valid.p, (size_t)M * hw * 4, cudaMemcpyDeviceToHost));
    return 0;
}

// avg_pool_2x2_kernel (main.cu:1150-1170) over [N][H][W].
int ref_pool(const float* in_h, float* out_h, long long N, int H, int W) {
    size_t nin = (size_t)N * H * W, nout = (size_t)N * (H / 2) * (W / 2);
    DBuf<float> in, out;
    RCHK(in.alloc(nin));
    RCHK(out.alloc(nout ? nout : 1));
    RCHK(cudaMemcpy(in.p, in_h, nin * 4, cudaMemcpyHostToDevice));
    int total = (int)nout;
    avg_pool_2x2_kernel<<<(total + 255) / 256, 256>>>(in.p, out.p, (int)N, H, W);
    RCHK(cudaGetLastError());
    RCHK(cudaMemcpy(out_h, out.p, nout * 4, cudaMemcpyDeviceToHost));
    return 0;
}

// batch_corr_sample_kernel x4 after a memset (main.cu:1597-1612).
// levels_h[l]: [M][hw][h>>l][w>>l]; coords_h [M][2][hw]; out_h [M][196][hw].
int ref_lookup_batched(const float* const* levels_h, const float* coords_h, float* out_h,
                       int M, int h, int w) {
    int hw = h * w;
    DBuf<float> lev[4], coords, out;
    for (int l = 0; l < 4; l++) {
        size_t n = (size_t)M * hw * (h >> l) * (w >> l);
        RCHK(lev[l].alloc(n ? n : 1));
        RCHK(cudaMemcpy(lev[l].p, levels_h[l], n * 4, cudaMemcpyHostToDevice));
    }
    RCHK(coords.alloc((size_t)M * 2 * hw));
    RCHK(cudaMemcpy(coords.p, coords_h, (size_t)M * 2 * hw * 4, cudaMemcpyHostToDevice));
    RCHK(out.alloc((size_t)M * 196 * hw));
    RCHK(cudaMemset(out.p, 0, (size_t)M * 196 * hw * 4));
    dim3 block(8, 8), grid((w + 7) / 8, (h + 7) / 8, M);
    for (int l = 0; l < 4; l++) {
        int ph = h >> l, pw = w >> l;
        float scale = 1.0f / (float)(1 << l);
        batch_corr_sample_kernel<<<grid, block>>>(lev[l].p, coords.p, out.p, M, 3, h, w, ph, pw,
                                                  hw, scale, l);
    }
    RCHK(cudaGetLastError());
    RCHK(cudaMemcpy(out_h, out.p, (size_t)M * 196 * hw * 4, cudaMemcpyDeviceToHost));
    return 0;
}

// corr_index_kernel x4, one edge (main.cu:1529-1552).
int ref_lookup_single(const float* const* levels_h, const float* coords_h, float* out_h, int h,
                      int w) {
    int hw = h * w, D = 7;
    DBuf<float> lev[4], coords, out;
    for (int l = 0; l < 4; l++) {
        size_t n = (size_t)hw * (h >> l) * (w >> l);
        RCHK(lev[l].alloc(n ? n : 1));
        RCHK(cudaMemcpy(lev[l].p, levels_h[l], n * 4, cudaMemcpyHostToDevice));
    }
    RCHK(coords.alloc(2 * (size_t)hw));
    RCHK(cudaMemcpy(coords.p, coords_h, 2 * (size_t)hw * 4, cudaMemcpyHostToDevice));
    RCHK(out.alloc(196 * (size_t)hw));
    dim3 block(8, 8), grid((w + 7) / 8, (h + 7) / 8);
    for (int l = 0; l < 4; l++) {
        float* level_out = out.p + (size_t)l * D * D * hw;
        RCHK(cudaMemset(level_out, 0, (size_t)D * D * hw * 4));
        corr_index_kernel<<<grid, block>>>(lev[l].p, coords.p, level_out, 3, h, w, h >> l,
                                           w >> l, 1.0f / (float)(1 << l));
    }
    RCHK(cudaGetLastError());
    RCHK(cudaMemcpy(out_h, out.p, 196 * (size_t)hw * 4, cudaMemcpyDeviceToHost));
    return 0;
}

// Whole batch_build_and_sample_correlation (main.cu:1555-1613), in chunks of 48
// edges like run_update_pass (main.cu:2185).  fmaps_h: [K][C=128][hw] fp32, rounded
// to fp16 on the device like DroidState::fmaps (main.cu:677).  If vol0_h is not
// NULL it receives the level-0 volume of every edge ([M][hw][hw]).
// iters > 0: additionally time `iters` repetitions of the chunk loop with inputs
// resident (after one warm-up pass) and store ms per repetition in *ms_out.
int ref_build_and_sample_fp16(const float* fmaps_h, int K, int h, int w, const int* ii,
                              const int* jj, int M, const float* coords_h, float alpha,
                              float* out_h, float* vol0_h, int iters, float* ms_out) {
    const int C = 128, CH = 48;
    int hw = h * w;
    size_t nf = (size_t)K * C * hw;
    DBuf<float> f32, vols, pyr[4], coords, out;
    DBuf<__half> fm;
    DBuf<void*> ptrs;
    RCHK(f32.alloc(nf));
    RCHK(fm.alloc(nf));
    RCHK(cudaMemcpy(f32.p, fmaps_h, nf * 4, cudaMemcpyHostToDevice));
    f32_to_f16<<<(unsigned)((nf + 255) / 256), 256>>>(f32.p, fm.p, nf);
    RCHK(vols.alloc((size_t)CH * hw * hw));
    for (int l = 1; l < 4; l++) RCHK(pyr[l].alloc((size_t)CH * hw * (h >> l) * (w >> l)));
    RCHK(coords.alloc((size_t)M * 2 * hw));
    RCHK(cudaMemcpy(coords.p, coords_h, (size_t)M * 2 * hw * 4, cudaMemcpyHostToDevice));
    RCHK(out.alloc((size_t)M * 196 * hw));
    RCHK(ptrs.alloc(3 * CH));
    cublasHandle_t cublas;
    BCHK(cublasCreate(&cublas));
    std::vector<void*> hp(3 * CH);

    auto chunk = [&](int bs, int e0, bool dump) -> int {
        for (int e = 0; e < bs; e++) {
            hp[e] = fm.p + (size_t)jj[e0 + e] * C * hw;           // A = fmaps[jj]
            hp[CH + e] = fm.p + (size_t)ii[e0 + e] * C * hw;      // B = fmaps[ii]
            hp[2 * CH + e] = vols.p + (size_t)e * hw * hw;
        }
        RCHK(cudaMemcpy(ptrs.p, hp.data(), 3 * CH * sizeof(void*), cudaMemcpyHostToDevice));
        float beta = 0.0f;
        BCHK(cublasGemmBatchedEx(cublas, CUBLAS_OP_N, CUBLAS_OP_T, hw, hw, 128, &alpha,
                                 (const void**)ptrs.p, CUDA_R_16F, hw,
                                 (const void**)(ptrs.p + CH), CUDA_R_16F, hw, &beta,
                                 (void**)(ptrs.p + 2 * CH), CUDA_R_32F, hw, bs,
                                 CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT_TENSOR_OP));
        int N1 = bs * hw;
        int total1 = N1 * (h / 2) * (w / 2);
        avg_pool_2x2_kernel<<<(total1 + 255) / 256, 256>>>(vols.p, pyr[1].p, N1, h, w);
        for (int l = 2; l < 4; l++) {
            int ph = h >> (l - 1), pw = w >> (l - 1);
            int totalL = N1 * (ph / 2) * (pw / 2);
            avg_pool_2x2_kernel<<<(totalL + 255) / 256, 256>>>(pyr[l - 1].p, pyr[l].p, N1, ph,
                                                                pw);
        }
        float* o = out.p + (size_t)e0 * 196 * hw;
        const float* c = coords.p + (size_t)e0 * 2 * hw;
        RCHK(cudaMemset(o, 0, (size_t)bs * 196 * hw * 4));
        dim3 block(8, 8), grid((w + 7) / 8, (h + 7) / 8, bs);
        for (int l = 0; l < 4; l++) {
            float* lv = (l == 0) ? vols.p : pyr[l].p;
            batch_corr_sample_kernel<<<grid, block>>>(lv, c, o, bs, 3, h, w, h >> l, w >> l, hw,
                                                      1.0f / (float)(1 << l), l);
        }
        RCHK(cudaGetLastError());
        if (dump)
            RCHK(cudaMemcpy(vol0_h + (size_t)e0 * hw * hw, vols.p, (size_t)bs * hw * hw * 4,
                            cudaMemcpyDeviceToHost));
        return 0;
    };
    auto pass = [&](bool dump) -> int {
        for (int e0 = 0; e0 < M; e0 += CH) {
            int bs = M - e0 < CH ? M - e0 : CH;
            int rc = chunk(bs, e0, dump);
            if (rc) return rc;
        }
        return 0;
    };
    int rc = pass(vol0_h != nullptr);
    if (rc) { cublasDestroy(cublas); return rc; }
    RCHK(cudaDeviceSynchronize());
    RCHK(cudaMemcpy(out_h, out.p, (size_t)M * 196 * hw * 4, cudaMemcpyDeviceToHost));
    if (iters > 0 && ms_out) {
        cudaEvent_t a, b;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        cudaEventRecord(a);
        for (int it = 0; it < iters && rc == 0; it++) rc = pass(false);
        cudaEventRecord(b);
        cudaEventSynchronize(b);
        float ms = 0;
        cudaEventElapsedTime(&ms, a, b);
        *ms_out = ms / iters;
        cudaEventDestroy(a);
        cudaEventDestroy(b);
    }
    cublasDestroy(cublas);
    return rc;
}

// GraphAgg scatter-mean exactly as the update step runs it (main.cu:2262-2294):
// a memset of the compact per-keyframe buffer, one scale_add_kernel launch
// (dst += 1 * src) per edge in edge order, then one launch (dst += (1/n - 1) * dst)
// per keyframe with n > 1 edges.  Compact order = ascending keyframe id
// (std::set).  feats_h [E][F]; agg_h [K][F], K = number of distinct ii_h.
int ref_scatter_mean(const float* feats_h, long long F, const int* ii_h, int E, float* agg_h,
                     int* K_out) {
    std::set<int> kf_set(ii_h, ii_h + E);
    std::vector<int> kfs(kf_set.begin(), kf_set.end());
    const int K = (int)kfs.size();
    std::map<int, int> compact;
    for (int i = 0; i < K; i++) compact[kfs[i]] = i;
    DBuf<float> feats, agg;
    RCHK(feats.alloc((size_t)E * F));
    RCHK(agg.alloc((size_t)K * F));
    RCHK(cudaMemcpy(feats.p, feats_h, (size_t)E * F * 4, cudaMemcpyHostToDevice));
    RCHK(cudaMemset(agg.p, 0, (size_t)K * F * 4));
    std::vector<int> count(K, 0);
    const int n = (int)F;
    for (int e = 0; e < E; e++) {
        const int c = compact[ii_h[e]];
        scale_add_kernel<<<(n + 255) / 256, 256>>>(agg.p + (size_t)c * F, feats.p + (size_t)e * F,
                                                   1.0f, n);
        count[c]++;
    }
    for (int i = 0; i < K; i++) {
        if (count[i] > 1) {
            float inv = 1.0f / (float)count[i];
            scale_add_kernel<<<(n + 255) / 256, 256>>>(agg.p + (size_t)i * F, agg.p + (size_t)i * F,
                                                       inv - 1.0f, n);
        }
    }
    RCHK(cudaGetLastError());
    RCHK(cudaDeviceSynchronize());
    RCHK(cudaMemcpy(agg_h, agg.p, (size_t)K * F * 4, cudaMemcpyDeviceToHost));
    if (K_out) *K_out = K;
    return 0;
}

}  // extern "C"

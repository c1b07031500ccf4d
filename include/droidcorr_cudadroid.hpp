// droidcorr_cudadroid.hpp -- header-only C++ shim that gives the correlation
// methods of slam-hands' CudaDroid (cuda_slam/main.cu:1499-1613, same methods at
// cuda_pipeline/slam.cuh:2796-2909) their original signatures on top of the C
// ABI in droidcorr.h.  A CudaDroid that owns one DroidCorrShim can forward
//
//   build_correlation(i, j)                        -> shim.build_correlation(i, j)
//   sample_correlation(coords_2hw, corr_out)       -> shim.sample_correlation(...)
//   batch_build_and_sample_correlation(M, e0, c, o)-> shim.batch_build_and_sample_correlation(...)
//
// and keep its buffers, edge lists (state.ii_host / jj_host) and layouts.  The
// shim owns the library context, the single-edge volume pyramid (corr_volume,
// corr_pyramid[1..3], main.cu:1323-1325) and a device copy of the edge lists.
// Errors are returned as DC_* status codes (the reference exited the process).
#ifndef DROIDCORR_CUDADROID_HPP_
#define DROIDCORR_CUDADROID_HPP_

#include <cuda_runtime.h>

#include <vector>

#include "droidcorr.h"

class DroidCorrShim {
public:
    // h, w: feature grid; max_kf: keyframe slots (DroidState::MAX_KEYFRAMES);
    // precision DC_PREC_FP16 reproduces the reference arithmetic.
    int init(int h, int w, int max_kf, int max_edges = 48, int precision = DC_PREC_FP16,
             float alpha = 1.0f / 16.0f) {
        dc_config cfg;
        dc_default_config(&cfg, h, w);
        cfg.max_frames = max_kf;
        cfg.max_edges = max_edges;
        cfg.precision = precision;
        cfg.alpha = alpha;
        h_ = h;
        w_ = w;
        int rc = dc_create(&cfg, &ctx_);
        if (rc) return rc;
        const size_t hw = (size_t)h * w;
        for (int l = 0; l < 4; l++) {
            const size_t n = hw * (size_t)(h >> l) * (size_t)(w >> l);
            if (cudaMalloc(&vol_[l], n * sizeof(float)) != cudaSuccess) return DC_ERR_NO_MEMORY;
        }
        if (cudaMalloc(&ii_dev_, max_edges * sizeof(int)) != cudaSuccess ||
            cudaMalloc(&jj_dev_, max_edges * sizeof(int)) != cudaSuccess)
            return DC_ERR_NO_MEMORY;
        return DC_OK;
    }
    ~DroidCorrShim() {
        for (int l = 0; l < 4; l++)
            if (vol_[l]) cudaFree(vol_[l]);
        if (ii_dev_) cudaFree(ii_dev_);
        if (jj_dev_) cudaFree(jj_dev_);
        dc_destroy(ctx_);
    }

    // After DroidState::add_keyframe wrote slot k of state.fmaps (__half [128][h][w]).
    int update_keyframe(const void* fmap_slot_dev, int slot, cudaStream_t s = 0) {
        return dc_set_frames(ctx_, fmap_slot_dev, DC_DTYPE_F16, slot, 1, s);
    }

    // CudaDroid::build_correlation(int i, int j), main.cu:1500.
    int build_correlation(int i, int j, cudaStream_t s = 0) {
        int e[2] = {i, j};
        if (cudaMemcpyAsync(ii_dev_, &e[0], sizeof(int), cudaMemcpyHostToDevice, s) ||
            cudaMemcpyAsync(jj_dev_, &e[1], sizeof(int), cudaMemcpyHostToDevice, s))
            return DC_ERR_CUDA;
        if (cudaStreamSynchronize(s) != cudaSuccess) return DC_ERR_CUDA;
        return dc_build_volume(ctx_, ii_dev_, jj_dev_, 1, vol_, s);
    }

    // CudaDroid::sample_correlation(float* coords_2hw, float* corr_out), main.cu:1529.
    int sample_correlation(const float* coords_2hw, float* corr_out, cudaStream_t s = 0) {
        return dc_lookup_single(ctx_, vol_, coords_2hw, corr_out, s);
    }

    // CudaDroid::batch_build_and_sample_correlation, main.cu:1555: edges
    // ii_host/jj_host[edge_start, edge_start + batch_size).
    int batch_build_and_sample_correlation(const std::vector<int>& ii_host,
                                           const std::vector<int>& jj_host, int batch_size,
                                           int edge_start, const float* coords_2hw,
                                           float* corr_out_196hw, cudaStream_t s = 0) {
        const size_t bytes = (size_t)batch_size * sizeof(int);
        if (cudaMemcpyAsync(ii_dev_, ii_host.data() + edge_start, bytes, cudaMemcpyHostToDevice, s) ||
            cudaMemcpyAsync(jj_dev_, jj_host.data() + edge_start, bytes, cudaMemcpyHostToDevice, s))
            return DC_ERR_CUDA;
        // the host vectors may change after return: finish the copies first
        if (cudaStreamSynchronize(s) != cudaSuccess) return DC_ERR_CUDA;
        return dc_build_and_lookup(ctx_, ii_dev_, jj_dev_, batch_size, coords_2hw,
                                   corr_out_196hw, s);
    }

    const float* corr_volume() const { return vol_[0]; }          // debug dump, main.cu:2859
    const float* corr_pyramid(int l) const { return vol_[l]; }
    dc_ctx* context() { return ctx_; }

private:
    dc_ctx* ctx_ = nullptr;
    float* vol_[4] = {nullptr, nullptr, nullptr, nullptr};
    int* ii_dev_ = nullptr;
    int* jj_dev_ = nullptr;
    int h_ = 0, w_ = 0;
};

#endif  // DROIDCORR_CUDADROID_HPP_

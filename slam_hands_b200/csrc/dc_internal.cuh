// dc_internal.cuh -- context and shared helpers of libdroidcorr (not installed).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "../../include/droidcorr.h"

#define DC_MAX_LEVELS 4
#define DC_MAX_RADIUS 3
#define DC_MAX_HW 16384

// Feature-map store: per slot and level, a pixel-major [rows_l][C] matrix of the
// precision's element type (float for FP32/TF32, __half for FP16,
// __nv_bfloat16 for BF16).  rows_l = hw_l rounded up to DC_ROW_PAD; the padding
// rows are zero.  All levels of all slots form one 2-D matrix
// [max_frames * frame_rows][C], so a (slot, level, pixel) row is
//   slot * frame_rows + level_row0[l] + pixel.
#define DC_ROW_PAD 128

struct dc_ctx {
    dc_config cfg;
    int device = 0;
    int hw = 0;
    int H[DC_MAX_LEVELS] = {0}, W[DC_MAX_LEVELS] = {0};
    long long level_row0[DC_MAX_LEVELS] = {0};
    long long frame_rows = 0;
    long long lo_rows = 0;  // DC_PREC_FP32X3: a slot holds hi rows, then the lo copy at +lo_rows
    int elem_bytes = 4;
    void* store = nullptr;  // device
    void* src_store = nullptr;  // another process's store, opened by dc_store_attach_source
    long long store_bytes = 0;
    long long other_bytes = 0;  // every other device allocation of the context (scratch, weights)
    int num_sms = 148;
    int max_ctas = 0;  // cap on the CTAs of the persistent fused kernel (0: one per SM)
    long long launches = 0;
    int* dev_err = nullptr;  // device error word raised by bounded device waits; the same
                             // allocation holds the scatter-mean lists from word 32 on
    // tensor map of the store for the tensor-core kernel (CUtensorMap storage)
    alignas(64) unsigned char tmap_a[128];
    // per level, a 4-D map [slot][H_l][W_l][C] of the same store with boxes of
    // 4 target rows x 8 target columns x 64 channels (the fused kernel's B boxes)
    alignas(64) unsigned char tmap_b[DC_MAX_LEVELS][128];
    alignas(64) unsigned char tmap_b_lo[DC_MAX_LEVELS][128];  // DC_PREC_FP32X3: the lo copy
    bool tc_ready = false;
    // fused kernel's tile order (dc_set_tile_order) and its scratch: the pixel
    // permutation [max_edges][hw] (tile position -> source pixel), one flag per
    // edge (1: permuted, 0: identity), the coordinates in tile-position order
    // [max_edges][2][hw]
    int tile_order = 0;
    int* tile_perm = nullptr;
    // 2-D map of the store with one-row boxes (row gathers of the source tile)
    alignas(64) unsigned char tmap_a_rows[128];
    // correlation encoder (dc_set_corr_encoder): packed fp16 weights, then the bias
    void* enc_w = nullptr;
    bool enc_ready = false;
    std::string err;
};

namespace dc {

// Per-level geometry passed by value to kernels.
struct Geom {
    int h, w, hw, C, levels, radius;
    int H[DC_MAX_LEVELS], W[DC_MAX_LEVELS];
    long long row0[DC_MAX_LEVELS];
    long long frame_rows;
    long long lo_rows;
    float alpha;
};

inline Geom geom_of(const dc_ctx* c) {
    Geom g;
    g.h = c->cfg.h;
    g.w = c->cfg.w;
    g.hw = c->hw;
    g.C = c->cfg.channels;
    g.levels = c->cfg.levels;
    g.radius = c->cfg.radius;
    for (int l = 0; l < DC_MAX_LEVELS; l++) {
        g.H[l] = c->H[l];
        g.W[l] = c->W[l];
        g.row0[l] = c->level_row0[l];
    }
    g.frame_rows = c->frame_rows;
    g.lo_rows = c->lo_rows;
    g.alpha = c->cfg.alpha;
    return g;
}

struct LevelPtrs {
    const float* p[DC_MAX_LEVELS];
};
struct LevelOutPtrs {
    float* p[DC_MAX_LEVELS];
};

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}

// fp32 -> tf32 value (round to nearest, ties away, 10 explicit mantissa bits),
// kept in an fp32 container.
__device__ __forceinline__ float round_tf32(float v) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return __uint_as_float(r);
}

// The bilinear combination of one output tap, in the reference's rounding order
// (batch_corr_sample_kernel, main.cu:1196-1213): the four contributions to
// output (a, b) arrive in loop order (i outer, j inner) -- taps (a,b), (a,b+1),
// (a+1,b), (a+1,b+1) -- each as fmaf(s * wx, wy, acc), starting from +0.
__device__ __forceinline__ float bilinear_tap(float acc, float s, bool valid, float wx,
                                              float wy) {
    return valid ? fmaf(s * wx, wy, acc) : acc;
}

}  // namespace dc

// Validate a configuration and fill the context's geometry (levels, store rows,
// element size, store bytes for `frames` slots).  Returns DC_OK or
// DC_ERR_INVALID_ARG.
int dc_init_geometry(dc_ctx* ctx, const dc_config& c, int frames);

// Store element type of a precision: 16-bit for the tensor-core precisions.
inline bool dc_store_is_16bit(int precision) { return precision != DC_PREC_FP32; }

// Launch helpers: record the launch and turn launch errors into a status.
int dc_fail(dc_ctx* ctx, int status, const std::string& msg);
int dc_check_launch(dc_ctx* ctx, const char* what);

// Kernel entry points implemented in the .cu files.
int dc_launch_store(dc_ctx* ctx, const void* fmaps, int dtype, int first, int count,
                    cudaStream_t s);
int dc_launch_store_zero_padding(dc_ctx* ctx, int first, int count, cudaStream_t s);
int dc_launch_volume_ffma(dc_ctx* ctx, const int* ii, const int* jj, int M, float* vol0,
                          cudaStream_t s);
int dc_launch_volume_tc(dc_ctx* ctx, const int* ii, const int* jj, int M, float* vol0,
                        cudaStream_t s);
int dc_launch_volume_pyramid(dc_ctx* ctx, float* const* vols, int M, cudaStream_t s);
int dc_launch_pool2x2(const float* in, float* out, long long N, int H, int W,
                      cudaStream_t s);
int dc_launch_lookup(dc_ctx* ctx, const float* const* vols, const float* coords, float* out,
                     int M, bool single_edge_arith, cudaStream_t s);
// A 2-D tensor map (CUtensorMap storage, 128 bytes) over a row-major fp32
// matrix [rows][cols] with boxes of box_rows x box_cols, no swizzle, elements
// outside the matrix read as zeros.  cols * 4 must be a multiple of 16.
int dc_tmap_2d_f32(void* tmap, const void* base, unsigned long long cols,
                   unsigned long long rows, unsigned box_cols, unsigned box_rows);
bool dc_tc_supported(const dc_ctx* ctx);
int dc_tc_prepare(dc_ctx* ctx);
int dc_launch_tc(dc_ctx* ctx, const int* ii, const int* jj, int M, const float* coords,
                 float* out, cudaStream_t s);
int dc_launch_project(dc_ctx* ctx, const float* poses, const float* disps,
                      const float* intrinsics, const int* ii, const int* jj, int M,
                      int num_frames, float* coords, float* valid, cudaStream_t s);
int dc_scatter_mean_impl(dc_ctx* ctx, const float* feats, long long F, const int* ii_host,
                         int E, float* agg, int* kf_ids_host, int* K_out, cudaStream_t s);
int dc_gather_rows_impl(dc_ctx* ctx, const float* src, long long F, int num_rows, const int* idx,
                        int n, float* dst, cudaStream_t s);
int dc_set_corr_encoder_impl(dc_ctx* ctx, const float* weight, const float* bias, int co,
                             cudaStream_t s);
int dc_launch_encoder(dc_ctx* ctx, const float* corr, int M, void* out, cudaStream_t s);
int dc_launch_alt(dc_ctx* ctx, const int* ii, const int* jj, int M, const float* coords,
                  float* out, cudaStream_t s);

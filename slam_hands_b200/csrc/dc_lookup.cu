// dc_lookup.cu -- radius-r bilinear lookup from materialised volumes.
//
// Replaces batch_corr_sample_kernel (cuda_slam/main.cu:1175-1217, one launch per
// level after a cudaMemset of the output, every tap a read-modify-write of
// global memory) and corr_index_kernel (main.cu:1079-1114, atomicAdd).  Here one
// thread owns one (edge, source pixel), walks all levels, keeps each output in a
// register and stores it once; consecutive threads own consecutive pixels, so
// every output channel is written with coalesced 128-byte stores.
//
// Arithmetic is the reference's, bit for bit: level-l coordinates are scaled by
// 2^-l before floor (main.cu:1189-1190); taps outside [0,H_l) x [0,W_l) add
// nothing; output (a, b) = channel a*D + b accumulates taps (a,b), (a,b+1),
// (a+1,b), (a+1,b+1) in that order as fmaf(s*wx, wy, acc) from +0 (nvcc's
// contraction of `out += s * wx * wy`).  The single-edge variant adds the
// rounded product (s*wx)*wy instead, as atomicAdd does.
#include "dc_internal.cuh"

namespace {

template <bool kSingle>
__device__ __forceinline__ float tap(float acc, float s, bool valid, float wx, float wy) {
    if (!valid) return acc;
    if (kSingle) return __fadd_rn(acc, __fmul_rn(__fmul_rn(s, wx), wy));
    return fmaf(__fmul_rn(s, wx), wy, acc);
}

template <bool kSingle, int R>
__global__ void __launch_bounds__(128) lookup_kernel(dc::LevelPtrs vols,
                                                     const float* __restrict__ coords,
                                                     float* __restrict__ out, dc::Geom g) {
    constexpr int D = 2 * R + 1, NW = 2 * R + 2;
    const int e = blockIdx.y;
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    const int hw = g.hw;
    if (p >= hw) return;
    const float cx = __ldg(coords + (size_t)e * 2 * hw + p);
    const float cy = __ldg(coords + (size_t)e * 2 * hw + hw + p);
    float* o = out + (size_t)e * g.levels * D * D * hw + p;
    for (int l = 0; l < g.levels; l++) {
        const int Hl = g.H[l], Wl = g.W[l];
        const float scale = 1.0f / (float)(1 << l);
        const float x0 = cx * scale, y0 = cy * scale;
        const float fx = floorf(x0), fy = floorf(y0);
        const float dx = x0 - fx, dy = y0 - fy;
        const int bx = (int)fx - R, by = (int)fy - R;
        const float* row = vols.p[l] + ((size_t)e * hw + p) * Hl * Wl;
        float s[NW][NW];  // s[i][j]: x offset i, y offset j
        bool vx[NW], vy[NW];
#pragma unroll
        for (int i = 0; i < NW; i++) {
            vx[i] = (unsigned)(bx + i) < (unsigned)Wl;
            vy[i] = (unsigned)(by + i) < (unsigned)Hl;
        }
#pragma unroll
        for (int j = 0; j < NW; j++)
#pragma unroll
            for (int i = 0; i < NW; i++)
                s[i][j] = (vx[i] && vy[j]) ? __ldg(row + (by + j) * Wl + (bx + i)) : 0.0f;
        const float ux = 1.0f - dx, uy = 1.0f - dy;
        float* ol = o + (size_t)l * D * D * hw;
#pragma unroll
        for (int a = 0; a < D; a++)
#pragma unroll
            for (int b = 0; b < D; b++) {
                float acc = 0.0f;
                acc = tap<kSingle>(acc, s[a][b], vx[a] && vy[b], ux, uy);
                acc = tap<kSingle>(acc, s[a][b + 1], vx[a] && vy[b + 1], ux, dy);
                acc = tap<kSingle>(acc, s[a + 1][b], vx[a + 1] && vy[b], dx, uy);
                acc = tap<kSingle>(acc, s[a + 1][b + 1], vx[a + 1] && vy[b + 1], dx, dy);
                __stcs(ol + (size_t)(a * D + b) * hw, acc);
            }
    }
}

template <bool kSingle>
int launch_r(dc_ctx* ctx, dc::LevelPtrs lp, const float* coords, float* out, int M,
             cudaStream_t s) {
    dc::Geom g = dc::geom_of(ctx);
    dim3 grid((g.hw + 127) / 128, M);
    switch (g.radius) {
        case 0: lookup_kernel<kSingle, 0><<<grid, 128, 0, s>>>(lp, coords, out, g); break;
        case 1: lookup_kernel<kSingle, 1><<<grid, 128, 0, s>>>(lp, coords, out, g); break;
        case 2: lookup_kernel<kSingle, 2><<<grid, 128, 0, s>>>(lp, coords, out, g); break;
        default: lookup_kernel<kSingle, 3><<<grid, 128, 0, s>>>(lp, coords, out, g); break;
    }
    return dc_check_launch(ctx, "lookup_kernel");
}

}  // namespace

int dc_launch_lookup(dc_ctx* ctx, const float* const* vols, const float* coords, float* out,
                     int M, bool single, cudaStream_t s) {
    dc::LevelPtrs lp;
    for (int l = 0; l < DC_MAX_LEVELS; l++) lp.p[l] = (l < ctx->cfg.levels) ? vols[l] : nullptr;
    return single ? launch_r<true>(ctx, lp, coords, out, M, s)
                  : launch_r<false>(ctx, lp, coords, out, M, s);
}

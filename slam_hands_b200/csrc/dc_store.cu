// dc_store.cu -- packing keyframe feature maps into the resident store.
//
// Input: the reference's per-keyframe layout [C][h][w] (DroidState::fmaps,
// cuda_slam/main.cu:677).  Output per slot: the map and its cascaded 2x2-average
// pyramid P_1..P_{L-1} (the same average as avg_pool_2x2_kernel,
// main.cu:1150-1170, applied to the map instead of the volume), pixel-major
// [pixels][C] in the precision's element type, so that one target pixel's
// channel vector is one contiguous row (coalesced gathers, K-major tensor-core
// operand tiles).
//
// One CTA packs one 8x8 tile of level-0 pixels of one slot.  With floor-pooling,
// every level-l cell lies inside exactly one such tile (cell (y, x) of level l
// covers level-0 rows [y 2^l, (y+1) 2^l), and 2^l divides 8), so tiles partition
// all levels and each map element is read from HBM once.
#include "dc_internal.cuh"

namespace {

// Packing modes: the value itself, its TF32 rounding, or (FP32X3) the fp16
// remainder x - fp16(x) for the lo copy.
enum { kPackPlain = 0, kPackTf32 = 1, kPackSplit = 2 };

template <typename T>
__device__ __forceinline__ T pack_value(float v, int mode) {
    if (mode == kPackTf32) v = dc::round_tf32(v);
    return dc::from_f32<T>(v);
}

// Writes element v of a row: the row itself, and under kPackSplit also the lo
// copy lo_off elements further (lo = fp16(x - fp16(x)), exact subtraction).
template <typename T>
__device__ __forceinline__ void put(T* dst, float v, int mode, long long lo_off) {
    const T hi = pack_value<T>(v, mode);
    dst[0] = hi;
    if (mode == kPackSplit) dst[lo_off] = dc::from_f32<T>(v - dc::to_f32(hi));
}

template <typename Tin, typename T>
__global__ void __launch_bounds__(256) store_pack_kernel(const Tin* __restrict__ fmaps,
                                                          T* __restrict__ store, dc::Geom g,
                                                          int first, int mode) {
    extern __shared__ float sm[];
    // one CTA: one 8x8 tile of one slot, 32 of the C channels
    constexpr int C = 32, lc = 5;
    const int CT = g.C;  // channels of a store row
    const int ngrp = CT / C;
    const int grp = blockIdx.z % ngrp;
    // per-channel rows padded by one float so that the channel-strided reads of
    // the pixel-major write-out hit distinct banks
    float* t0 = sm;             // [C][65]  level 0, tile-local (ty*8+tx)
    float* t1 = t0 + C * 65;    // [C][17]  level 1
    float* t2 = t1 + C * 17;    // [C][5]   level 2
    float* t3 = t2 + C * 5;     // [C][1]   level 3
    const int slot_local = blockIdx.z / ngrp;
    const int slot = first + slot_local;
    const int x0 = blockIdx.x * 8, y0 = blockIdx.y * 8;
    const Tin* f = fmaps + ((size_t)slot_local * CT + grp * C) * g.hw;
    T* st = store + (size_t)slot * g.frame_rows * CT + grp * C;
    const long long lo_off = g.lo_rows * CT;

    // all loads of a thread in flight at once (8 per thread)
    static_assert(C * 64 % 256 == 0, "256 threads");
    float lv[C * 64 / 256];
#pragma unroll
    for (int it = 0; it < C * 64 / 256; it++) {
        const int idx = threadIdx.x + 256 * it;
        const int c = idx >> 6, k = idx & 63;
        const int y = y0 + (k >> 3), x = x0 + (k & 7);
        lv[it] = (y < g.h && x < g.w) ? dc::to_f32(f[(size_t)c * g.hw + y * g.w + x]) : 0.0f;
    }
#pragma unroll
    for (int it = 0; it < C * 64 / 256; it++) {
        const int idx = threadIdx.x + 256 * it;
        t0[(idx >> 6) * 65 + (idx & 63)] = lv[it];
    }
    __syncthreads();
    // level 0 rows
#pragma unroll
    for (int idx = threadIdx.x; idx < C * 64; idx += 256) {
        int k = idx >> lc, c = idx & (C - 1);
        int y = y0 + (k >> 3), x = x0 + (k & 7);
        if (y < g.h && x < g.w)
            put<T>(st + (g.row0[0] + y * g.w + x) * CT + c, t0[c * 65 + k], mode, lo_off);
    }
    // cascaded pooling inside the tile: level l has (8 >> l)^2 tile-local cells
    float* src = t0;
    float* dstv[3] = {t1, t2, t3};
    for (int l = 1; l < g.levels; l++) {
        const int sw = 8 >> (l - 1), dw = 8 >> l;  // tile-local widths
        const int ld = 3 - l;                        // log2(dw)
        float* dst = dstv[l - 1];
        for (int idx = threadIdx.x; idx < C * dw * dw; idx += blockDim.x) {
            int c = idx >> (2 * ld), k = idx & (dw * dw - 1);
            int ly = k >> ld, lx = k & (dw - 1);
            const float* s = src + c * (sw * sw + (sw > 1));
            float v = s[(2 * ly) * sw + 2 * lx] + s[(2 * ly) * sw + 2 * lx + 1];
            v = v + s[(2 * ly + 1) * sw + 2 * lx];
            v = v + s[(2 * ly + 1) * sw + 2 * lx + 1];
            dst[c * (dw * dw + (dw > 1)) + k] = 0.25f * v;
        }
        __syncthreads();
        const int gy0 = y0 >> l, gx0 = x0 >> l;
        for (int idx = threadIdx.x; idx < C * dw * dw; idx += blockDim.x) {
            int k = idx >> lc, c = idx & (C - 1);
            int y = gy0 + (k >> ld), x = gx0 + (k & (dw - 1));
            if (y < g.H[l] && x < g.W[l])
                put<T>(st + (g.row0[l] + y * g.W[l] + x) * CT + c, dst[c * (dw * dw + (dw > 1)) + k],
                       mode, lo_off);
        }
        src = dst;
    }
}

template <typename Tin, typename T>
int launch_store_t(dc_ctx* ctx, const void* fmaps, int first, int count, cudaStream_t s) {
    dc::Geom g = dc::geom_of(ctx);
    dim3 grid((g.w + 7) / 8, (g.h + 7) / 8, count * (g.C / 32));
    size_t smem = (size_t)32 * (65 + 17 + 5 + 1) * sizeof(float);
    auto k = store_pack_kernel<Tin, T>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const int mode = ctx->cfg.precision == DC_PREC_TF32    ? kPackTf32
                     : ctx->cfg.precision == DC_PREC_FP32X3 ? kPackSplit
                                                            : kPackPlain;
    k<<<grid, 256, smem, s>>>((const Tin*)fmaps, (T*)ctx->store, g, first, mode);
    return dc_check_launch(ctx, "store_pack_kernel");
}

// Zeroes the padding rows of store slots first .. first + count - 1: per level,
// rows hw_l .. rows_l - 1 (rows_l = hw_l rounded up to DC_ROW_PAD), which the
// tensor-core kernels read as operand rows and must hold zeros.  One CTA per
// (slot, level); 16-byte stores.
__global__ void __launch_bounds__(256) store_zero_padding_kernel(uint4* __restrict__ store,
                                                                  dc::Geom g, int first,
                                                                  int row_bytes) {
    const int l = blockIdx.y, slot = first + blockIdx.x;
    const long long hw_l = (long long)g.H[l] * g.W[l];
    const long long rows_l = (hw_l + DC_ROW_PAD - 1) / DC_ROW_PAD * DC_ROW_PAD;
    // blockIdx.z = 1: the lo copy of an FP32X3 slot
    const long long r0 = (long long)slot * g.frame_rows + blockIdx.z * g.lo_rows + g.row0[l] + hw_l;
    const long long n16 = (rows_l - hw_l) * row_bytes / 16;
    uint4* p = store + r0 * row_bytes / 16;
    for (long long i = threadIdx.x; i < n16; i += blockDim.x) p[i] = make_uint4(0, 0, 0, 0);
}

}  // namespace

int dc_launch_store_zero_padding(dc_ctx* ctx, int first, int count, cudaStream_t s) {
    if (count <= 0) return DC_OK;
    dim3 grid(count, ctx->cfg.levels, ctx->lo_rows > 0 ? 2 : 1);
    store_zero_padding_kernel<<<grid, 256, 0, s>>>(static_cast<uint4*>(ctx->store),
                                                  dc::geom_of(ctx), first,
                                                  ctx->cfg.channels * ctx->elem_bytes);
    return dc_check_launch(ctx, "store_zero_padding_kernel");
}

int dc_launch_store(dc_ctx* ctx, const void* fmaps, int dtype, int first, int count,
                    cudaStream_t s) {
    const int p = ctx->cfg.precision;
    // store element: bf16 for BF16, fp32 for FP32, fp16 otherwise (FP16, TF32, FP32X3)
    if (dtype == DC_DTYPE_F32) {
        if (p == DC_PREC_BF16) return launch_store_t<float, __nv_bfloat16>(ctx, fmaps, first, count, s);
        if (p == DC_PREC_FP32) return launch_store_t<float, float>(ctx, fmaps, first, count, s);
        return launch_store_t<float, __half>(ctx, fmaps, first, count, s);
    }
    if (p == DC_PREC_BF16) return launch_store_t<__half, __nv_bfloat16>(ctx, fmaps, first, count, s);
    if (p == DC_PREC_FP32) return launch_store_t<__half, float>(ctx, fmaps, first, count, s);
    return launch_store_t<__half, __half>(ctx, fmaps, first, count, s);
}

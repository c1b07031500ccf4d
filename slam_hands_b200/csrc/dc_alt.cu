// dc_alt.cu -- on-the-fly ("alt-corr") lookup: per-pixel gathered dot products
// against the pooled target maps of the store, no volume.
//
// For edge e, source pixel p and level l the lookup needs the volume values
// V_l[p][q] = alpha * <f_ii[:, p], P_l f_jj[:, q]> only at the (2r+2)^2 taps of
// its window.  One warp owns one (pixel, level) at a time: lane k holds channels
// [k*CPL, (k+1)*CPL) of f_ii[:, p] in registers, reads the same channels of each
// tap's target vector (one coalesced C-element row of the pixel-major store) and
// keeps per-tap partial sums for 32 taps at a time (the window's two halves).
// A transposed butterfly then reduces the 32 partials across the 32 lanes in 31
// shuffles (instead of 32 x 5), leaving tap k in lane k.  The bilinear combination uses the reference's rounding
// order (batch_corr_sample_kernel, cuda_slam/main.cu:1196-1213).
//
// A CTA owns one edge and 32 consecutive source pixels; its 8 warps take 4
// pixels each and stage the 196 outputs in shared memory, which the CTA then
// writes as coalesced 128-byte rows of [196][hw].
#include "dc_internal.cuh"

namespace {

constexpr int kPix = 32;    // pixels per CTA
constexpr int kWarps = 8;

template <typename T, int CPL>
__device__ __forceinline__ void load_ch(const T* p, float (&v)[CPL]) {
    if constexpr (sizeof(T) == 4) {
        if constexpr (CPL == 1) {
            v[0] = __ldg(reinterpret_cast<const float*>(p));
        } else if constexpr (CPL == 2) {
            float2 t = __ldg(reinterpret_cast<const float2*>(p));
            v[0] = t.x; v[1] = t.y;
        } else {
#pragma unroll
            for (int k = 0; k < CPL / 4; k++) {
                float4 t = __ldg(reinterpret_cast<const float4*>(p) + k);
                v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < CPL; k++) v[k] = dc::to_f32(p[k]);
    }
}

// Transposed butterfly: on entry each lane has 32 partial sums x[0..31] (one per
// tap); on exit lane k holds the full sum of tap k in x[0] (31 shuffles instead
// of 32 x 5).
__device__ __forceinline__ void reduce32(float (&x)[32], int lane) {
#pragma unroll
    for (int step = 0; step < 5; step++) {
        const int half = 16 >> step;  // live entries after this step
        const int bit = 16 >> step;   // partner distance
        const bool upper = (lane & bit) != 0;
#pragma unroll
        for (int i = 0; i < half; i++) {
            float mine = upper ? x[half + i] : x[i];
            float other = upper ? x[i] : x[half + i];
            x[i] = mine + __shfl_xor_sync(0xffffffffu, other, bit);
        }
    }
}

template <typename T, int CPL, int R>
__global__ void __launch_bounds__(kWarps * 32) alt_lookup_kernel(
    const T* __restrict__ store, const int* __restrict__ ii, const int* __restrict__ jj,
    int max_frames, const float* __restrict__ coords, float* __restrict__ out, dc::Geom g) {
    constexpr int D = 2 * R + 1, NW = 2 * R + 2;
    extern __shared__ float sm[];
    const int nch = g.levels * D * D;
    float* sout = sm;                                // [nch][kPix + 1]
    float* swin = sm + nch * (kPix + 1);             // [kWarps][64]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.y;
    const int pbase = blockIdx.x * kPix;
    const int hw = g.hw, C = g.C;
    const int si = ii[e], sj = jj[e];
    const bool ok = si >= 0 && si < max_frames && sj >= 0 && sj < max_frames;
    float* win = swin + warp * 64;

    for (int pi = warp; pi < kPix; pi += kWarps) {
        const int p = pbase + pi;
        if (p >= hw) break;
        const float cx = __ldg(coords + (size_t)e * 2 * hw + p);
        const float cy = __ldg(coords + (size_t)e * 2 * hw + hw + p);
        float a[CPL];
        if (ok) load_ch<T, CPL>(store + ((size_t)si * g.frame_rows + g.row0[0] + p) * C + lane * CPL, a);
        for (int l = 0; l < g.levels; l++) {
            const int Hl = g.H[l], Wl = g.W[l];
            const float scale = 1.0f / (float)(1 << l);
            const float x0 = cx * scale, y0 = cy * scale;
            const float fx = floorf(x0), fy = floorf(y0);
            const float dx = x0 - fx, dy = y0 - fy;
            const int bx = (int)fx - R, by = (int)fy - R;
            const T* tgt = store + ((size_t)sj * g.frame_rows + g.row0[l]) * C + lane * CPL;
            // the 8x8 window in two halves of 32 taps (x offsets 0-3, then 4-7):
            // half the live partial sums, twice the resident warps
#pragma unroll
            for (int hf = 0; hf < 2; hf++) {
                float part[32];
#pragma unroll
                for (int kk = 0; kk < 32; kk++) {
                    const int k = 32 * hf + kk;
                    const int i = k >> 3, j = k & 7;  // x offset i, y offset j
                    part[kk] = 0.0f;
                    if (i < NW && j < NW && ok) {
                        const int x1 = bx + i, y1 = by + j;
                        if ((unsigned)x1 < (unsigned)Wl && (unsigned)y1 < (unsigned)Hl) {
                            float b[CPL];
                            load_ch<T, CPL>(tgt + (size_t)(y1 * Wl + x1) * C, b);
                            float s = 0.0f;
#pragma unroll
                            for (int c = 0; c < CPL; c++) s = fmaf(a[c], b[c], s);
                            part[kk] = s;
                        }
                    }
                }
                reduce32(part, lane);
                win[32 * hf + lane] = g.alpha * part[0];
            }
            __syncwarp();
            const float ux = 1.0f - dx, uy = 1.0f - dy;
            for (int o = lane; o < D * D; o += 32) {
                const int aa = o / D, bb = o % D;
                const bool vx0 = (unsigned)(bx + aa) < (unsigned)Wl;
                const bool vx1 = (unsigned)(bx + aa + 1) < (unsigned)Wl;
                const bool vy0 = (unsigned)(by + bb) < (unsigned)Hl;
                const bool vy1 = (unsigned)(by + bb + 1) < (unsigned)Hl;
                float acc = 0.0f;
                acc = dc::bilinear_tap(acc, win[aa * 8 + bb], vx0 && vy0, ux, uy);
                acc = dc::bilinear_tap(acc, win[aa * 8 + bb + 1], vx0 && vy1, ux, dy);
                acc = dc::bilinear_tap(acc, win[(aa + 1) * 8 + bb], vx1 && vy0, dx, uy);
                acc = dc::bilinear_tap(acc, win[(aa + 1) * 8 + bb + 1], vx1 && vy1, dx, dy);
                sout[(l * D * D + o) * (kPix + 1) + pi] = acc;
            }
            __syncwarp();
        }
    }
    __syncthreads();
    float* oe = out + (size_t)e * nch * hw;
    for (int idx = threadIdx.x; idx < nch * kPix; idx += blockDim.x) {
        const int ch = idx / kPix, pi = idx % kPix;
        const int p = pbase + pi;
        if (p < hw) __stcs(oe + (size_t)ch * hw + p, sout[ch * (kPix + 1) + pi]);
    }
}

template <typename T, int CPL>
int launch_t(dc_ctx* ctx, const int* ii, const int* jj, int M, const float* coords, float* out,
             cudaStream_t s) {
    dc::Geom g = dc::geom_of(ctx);
    const int D = 2 * g.radius + 1;
    size_t smem = ((size_t)g.levels * D * D * (kPix + 1) + kWarps * 64) * sizeof(float);
    dim3 grid((g.hw + kPix - 1) / kPix, M);
    const T* st = (const T*)ctx->store;
    const int mf = ctx->cfg.max_frames;
#define DC_ALT_LAUNCH(RR)                                                                     \
    do {                                                                                      \
        auto k = alt_lookup_kernel<T, CPL, RR>;                                               \
        if (smem > 48 * 1024)                                                                 \
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);  \
        k<<<grid, kWarps * 32, smem, s>>>(st, ii, jj, mf, coords, out, g);                    \
    } while (0)
    switch (g.radius) {
        case 0: DC_ALT_LAUNCH(0); break;
        case 1: DC_ALT_LAUNCH(1); break;
        case 2: DC_ALT_LAUNCH(2); break;
        default: DC_ALT_LAUNCH(3); break;
    }
#undef DC_ALT_LAUNCH
    return dc_check_launch(ctx, "alt_lookup_kernel");
}

template <typename T>
int launch_c(dc_ctx* ctx, const int* ii, const int* jj, int M, const float* coords, float* out,
             cudaStream_t s) {
    switch (ctx->cfg.channels / 32) {
        case 1: return launch_t<T, 1>(ctx, ii, jj, M, coords, out, s);
        case 2: return launch_t<T, 2>(ctx, ii, jj, M, coords, out, s);
        case 4: return launch_t<T, 4>(ctx, ii, jj, M, coords, out, s);
        case 8: return launch_t<T, 8>(ctx, ii, jj, M, coords, out, s);
    }
    return dc_fail(ctx, DC_ERR_UNSUPPORTED, "channels must be 32, 64, 128 or 256");
}

}  // namespace

int dc_launch_alt(dc_ctx* ctx, const int* ii, const int* jj, int M, const float* coords,
                  float* out, cudaStream_t s) {
    switch (ctx->cfg.precision) {
        case DC_PREC_FP16:
        case DC_PREC_TF32:  // TF32-rounded values held as fp16
            return launch_c<__half>(ctx, ii, jj, M, coords, out, s);
        case DC_PREC_BF16: return launch_c<__nv_bfloat16>(ctx, ii, jj, M, coords, out, s);
        default: return launch_c<float>(ctx, ii, jj, M, coords, out, s);
    }
}

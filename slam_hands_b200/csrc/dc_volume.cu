// dc_volume.cu -- materialised correlation volumes and their pyramid.
//
//   volume_ffma_kernel    V0[e][p][q] = alpha * sum_c f_ii[c][p] f_jj[c][q]
//                         (the cublasGemmBatchedEx of cuda_slam/main.cu:1573-1581,
//                         as exact fp32 FFMA: one fmaf chain over c = 0..C-1 per
//                         output, then one multiply by alpha).
//   volume_pyramid_kernel V_l = 2x2 average of V_{l-1} over the target axes,
//                         cascaded (avg_pool_2x2_kernel x3, main.cu:1586-1595),
//                         all levels from one read of each V0 row.
//   pool2x2_kernel        one level of avg_pool_2x2_kernel (main.cu:1150-1170).
//
// The volume build writes hw^2 fp32 per edge and reads 2 hw C inputs, so it is
// HBM-store bound on B200 (about 60 flop per byte at C = 128).
#include "dc_internal.cuh"

namespace {

constexpr int BT = 128;  // output tile (p and q)
constexpr int BK = 8;    // channels per stage

template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&v)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&v)[4]) {
    float4 t = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
template <>
__device__ __forceinline__ void load4<__half>(const __half* p, float (&v)[4]) {
    uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
    float2 a = __half22float2(*reinterpret_cast<__half2*>(&t.x));
    float2 b = __half22float2(*reinterpret_cast<__half2*>(&t.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
    uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
    float2 a = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&t.x));
    float2 b = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&t.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

// 256 threads; thread (tx, ty) owns rows {ty*4+i, 64+ty*4+i} and columns
// {tx*4+j, 64+tx*4+j} of the 128x128 tile.
template <typename T>
__global__ void __launch_bounds__(256) volume_ffma_kernel(const T* __restrict__ store,
                                                           const int* __restrict__ ii,
                                                           const int* __restrict__ jj,
                                                           int max_frames, dc::Geom g,
                                                           float* __restrict__ vol0) {
    __shared__ __align__(16) float As[2][BK][BT];
    __shared__ __align__(16) float Bs[2][BK][BT];
    const int e = blockIdx.z;
    const int q0 = blockIdx.x * BT, p0 = blockIdx.y * BT;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int hw = g.hw, C = g.C;
    const int si = ii[e], sj = jj[e];
    float* V = vol0 + (size_t)e * hw * hw;
    const bool ok = si >= 0 && si < max_frames && sj >= 0 && sj < max_frames;

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;

    if (ok) {
        const T* A = store + (size_t)si * g.frame_rows * C;  // level 0 rows of ii
        const T* B = store + (size_t)sj * g.frame_rows * C;
        // loader: thread -> (pixel r = tid >> 1, channels c4 = (tid & 1) * 4 .. +3)
        const int lr = tid >> 1, lc = (tid & 1) * 4;
        const bool pa = p0 + lr < hw, pb = q0 + lr < hw;
        float ra[4], rb[4];
        auto fetch = [&](int k0) {
            if (pa) load4<T>(A + (size_t)(p0 + lr) * C + k0 + lc, ra);
            else ra[0] = ra[1] = ra[2] = ra[3] = 0.0f;
            if (pb) load4<T>(B + (size_t)(q0 + lr) * C + k0 + lc, rb);
            else rb[0] = rb[1] = rb[2] = rb[3] = 0.0f;
        };
        auto stash = [&](int buf) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                As[buf][lc + i][lr] = ra[i];
                Bs[buf][lc + i][lr] = rb[i];
            }
        };
        fetch(0);
        stash(0);
        __syncthreads();
        const int nk = C / BK;
        for (int kt = 0; kt < nk; kt++) {
            const int buf = kt & 1;
            if (kt + 1 < nk) fetch((kt + 1) * BK);
#pragma unroll
            for (int k = 0; k < BK; k++) {
                float a[8], b[8];
                float4 t;
                t = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
                a[0] = t.x; a[1] = t.y; a[2] = t.z; a[3] = t.w;
                t = *reinterpret_cast<const float4*>(&As[buf][k][64 + ty * 4]);
                a[4] = t.x; a[5] = t.y; a[6] = t.z; a[7] = t.w;
                t = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
                b[0] = t.x; b[1] = t.y; b[2] = t.z; b[3] = t.w;
                t = *reinterpret_cast<const float4*>(&Bs[buf][k][64 + tx * 4]);
                b[4] = t.x; b[5] = t.y; b[6] = t.z; b[7] = t.w;
#pragma unroll
                for (int i = 0; i < 8; i++)
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
            }
            if (kt + 1 < nk) {
                stash(buf ^ 1);
                __syncthreads();
            }
        }
    }
    const bool vec = (hw & 3) == 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int p = p0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (p >= hw) continue;
        float* row = V + (size_t)p * hw;
#pragma unroll
        for (int half = 0; half < 2; half++) {
            const int q = q0 + half * 64 + tx * 4;
            float o[4];
#pragma unroll
            for (int j = 0; j < 4; j++) o[j] = g.alpha * acc[i][half * 4 + j];
            if (vec && q + 3 < hw) {
                *reinterpret_cast<float4*>(row + q) = make_float4(o[0], o[1], o[2], o[3]);
            } else {
                for (int j = 0; j < 4; j++)
                    if (q + j < hw) row[q + j] = o[j];
            }
        }
    }
}

// One 2x2 average in the reference's rounding order: 0.25f * (((a + b) + c) + d).
__device__ __forceinline__ float avg4(float a, float b, float c, float d) {
    return 0.25f * (__fadd_rn(__fadd_rn(__fadd_rn(a, b), c), d));
}

// Coarser levels of one volume row from its level-0 map in shared memory (the
// levels lie back to back from sm).
__device__ __forceinline__ void pyramid_levels(float* sm, const dc::LevelOutPtrs& vols,
                                               long long row, const dc::Geom& g) {
    const float* s = sm;
    float* d = sm + g.H[0] * g.W[0];
#pragma unroll
    for (int l = 1; l < DC_MAX_LEVELS; l++) {
        if (l >= g.levels) break;
        const int Ws = g.W[l - 1], Wd = g.W[l], nd = g.H[l] * g.W[l];
        float* out = vols.p[l] ? vols.p[l] + (size_t)row * nd : nullptr;
        for (int i = threadIdx.x; i < nd; i += blockDim.x) {
            const int y = i / Wd, x = i - y * Wd;
            const float v = avg4(s[(2 * y) * Ws + 2 * x], s[(2 * y) * Ws + 2 * x + 1],
                                 s[(2 * y + 1) * Ws + 2 * x], s[(2 * y + 1) * Ws + 2 * x + 1]);
            d[i] = v;
            if (out) out[i] = v;
        }
        __syncthreads();
        s = d;
        d += nd;
    }
}

// Grid-stride over volume rows; each row's level-0 map goes through shared
// memory once and all coarser levels are produced from it.  With rows of a
// multiple of 4 floats, every thread holds KV float4 of the NEXT row in
// registers while the current row is pooled and stored, so each SM keeps its
// rows' reads in flight (HBM-bound: one read of V0, one write of V1..V3).
template <int KV>
__global__ void __launch_bounds__(256) volume_pyramid_kernel(dc::LevelOutPtrs vols, long long N,
                                                              dc::Geom g) {
    extern __shared__ float sm[];
    const int n0 = g.H[0] * g.W[0];
    if (KV > 0) {
        const int nv = n0 / 4;
        float4 r[KV > 0 ? KV : 1];
        long long row = blockIdx.x;
#define DC_PYR_FETCH(ROW)                                                                 \
    do {                                                                                  \
        const float4* src_ = reinterpret_cast<const float4*>(vols.p[0] + (size_t)(ROW) * n0); \
        _Pragma("unroll") for (int k = 0; k < KV; k++) {                                  \
            const int idx = threadIdx.x + k * blockDim.x;                                 \
            if (idx < nv) r[k] = __ldcs(src_ + idx);                                      \
        }                                                                                 \
    } while (0)
        if (row < N) DC_PYR_FETCH(row);
        for (; row < N; row += gridDim.x) {
#pragma unroll
            for (int k = 0; k < KV; k++) {
                const int idx = threadIdx.x + k * blockDim.x;
                if (idx < nv) reinterpret_cast<float4*>(sm)[idx] = r[k];
            }
            __syncthreads();
            if (row + gridDim.x < N) DC_PYR_FETCH(row + gridDim.x);  // in flight while pooling
            pyramid_levels(sm, vols, row, g);
        }
#undef DC_PYR_FETCH
    } else {
        for (long long row = blockIdx.x; row < N; row += gridDim.x) {
            const float* src = vols.p[0] + (size_t)row * n0;
            for (int i = threadIdx.x; i < n0; i += blockDim.x) sm[i] = __ldcs(src + i);
            __syncthreads();
            pyramid_levels(sm, vols, row, g);
        }
    }
}

__global__ void pool2x2_kernel(const float* __restrict__ in, float* __restrict__ out,
                               long long total, int H, int W) {
    const int oH = H / 2, oW = W / 2;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        long long n = idx / (oH * oW);
        int rem = (int)(idx % (oH * oW));
        int oy = rem / oW, ox = rem % oW;
        const float* s = in + (size_t)n * H * W + (2 * oy) * W + 2 * ox;
        out[idx] = avg4(s[0], s[1], s[W], s[W + 1]);
    }
}

}  // namespace

int dc_launch_volume_ffma(dc_ctx* ctx, const int* ii, const int* jj, int M, float* vol0,
                          cudaStream_t s) {
    dc::Geom g = dc::geom_of(ctx);
    dim3 grid((g.hw + BT - 1) / BT, (g.hw + BT - 1) / BT, M);
    switch (ctx->cfg.precision) {
        case DC_PREC_FP16:
        case DC_PREC_TF32:
            volume_ffma_kernel<__half><<<grid, 256, 0, s>>>((const __half*)ctx->store, ii, jj,
                                                            ctx->cfg.max_frames, g, vol0);
            break;
        case DC_PREC_BF16:
            volume_ffma_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
                (const __nv_bfloat16*)ctx->store, ii, jj, ctx->cfg.max_frames, g, vol0);
            break;
        default:
            volume_ffma_kernel<float><<<grid, 256, 0, s>>>((const float*)ctx->store, ii, jj,
                                                           ctx->cfg.max_frames, g, vol0);
    }
    return dc_check_launch(ctx, "volume_ffma_kernel");
}

int dc_launch_volume_pyramid(dc_ctx* ctx, float* const* vols, int M, cudaStream_t s) {
    dc::Geom g = dc::geom_of(ctx);
    if (g.levels < 2) return DC_OK;
    bool any = false;
    dc::LevelOutPtrs lp;
    for (int l = 0; l < DC_MAX_LEVELS; l++) {
        lp.p[l] = (l < g.levels) ? vols[l] : nullptr;
        if (l > 0 && lp.p[l]) any = true;
    }
    if (!any) return DC_OK;
    // A NULL level still has to be formed (in shared memory) if a coarser one is
    // requested; the kernel only skips the store.
    size_t smem = 0;
    for (int l = 0; l < DC_MAX_LEVELS; l++) smem += (size_t)g.H[l] * g.W[l] * sizeof(float);
    long long N = (long long)M * g.hw;
    const int n0 = g.H[0] * g.W[0];
    // float4 per thread of one row (256 threads), rounded up to an instantiation
    const int kv = (n0 & 3) ? 0 : (n0 / 4 + 255) / 256;
    // persistent: as many CTAs as fit on the device at once
#define DC_PYR_LAUNCH(KV)                                                                 \
    do {                                                                                  \
        if (smem > 48 * 1024)                                                             \
            cudaFuncSetAttribute(volume_pyramid_kernel<KV>,                               \
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
        int per_sm = 0;                                                                   \
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, volume_pyramid_kernel<KV>, \
                                                      256, smem);                         \
        long long blocks = (long long)ctx->num_sms * (per_sm > 0 ? per_sm : 1);           \
        if (blocks > N) blocks = N;                                                       \
        volume_pyramid_kernel<KV><<<(unsigned)blocks, 256, smem, s>>>(lp, N, g);          \
    } while (0)
    if (kv == 0) DC_PYR_LAUNCH(0);
    else if (kv <= 1) DC_PYR_LAUNCH(1);
    else if (kv <= 2) DC_PYR_LAUNCH(2);
    else if (kv <= 3) DC_PYR_LAUNCH(3);
    else if (kv <= 4) DC_PYR_LAUNCH(4);
    else if (kv <= 6) DC_PYR_LAUNCH(6);
    else if (kv <= 8) DC_PYR_LAUNCH(8);
    else if (kv <= 12) DC_PYR_LAUNCH(12);
    else DC_PYR_LAUNCH(16);
#undef DC_PYR_LAUNCH
    return dc_check_launch(ctx, "volume_pyramid_kernel");
}

int dc_launch_pool2x2(const float* in, float* out, long long N, int H, int W, cudaStream_t s) {
    long long total = N * (H / 2) * (W / 2);
    if (total == 0) return DC_OK;
    long long blocks = (total + 255) / 256;
    if (blocks > 148LL * 64) blocks = 148LL * 64;
    pool2x2_kernel<<<(unsigned)blocks, 256, 0, s>>>(in, out, total, H, W);
    return cudaGetLastError() == cudaSuccess ? DC_OK : DC_ERR_CUDA;
}

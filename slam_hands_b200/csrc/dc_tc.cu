// dc_tc.cu -- fused build + pyramid + lookup on the 5th-generation tensor cores.
//
// Drop-in for CudaDroid::batch_build_and_sample_correlation
// (cuda_slam/main.cu:1555-1613) that never writes a volume.  For one edge e and
// one tile of 128 source pixels p, the lookup needs, per level l, the volume
// values V_l[p][q] = alpha * <f_ii[:, p], P_l f_jj[:, q]> at the (2r+2)^2 taps
// around each pixel's scaled coordinate.  The CTA
//   1. reduces, over its 128 pixels, the range of target rows any window of
//      level l touches (so only those rows of the level are correlated);
//   2. streams those rows of the pooled target map P_l f_jj (pixel-major store,
//      K-major operand) through shared memory with TMA, 256 target pixels per
//      chunk, double-buffered;
//   3. computes the 128 x 256 x C correlation chunk with tcgen05.mma (kind::f16,
//      fp16 or bf16 operands, fp32 accumulation in TMEM, two accumulators so the
//      epilogue of chunk c overlaps the MMAs of chunk c+1);
//   4. reads back only the 32-column TMEM slices that hold some pixel's window
//      taps (tcgen05.ld), picks each pixel's taps into its window in shared
//      memory, and after the last chunk of a level forms the (2r+1)^2 bilinear
//      outputs in the reference's rounding order (main.cu:1196-1213) and stores
//      them with coalesced 128-byte rows of out[e][l*(2r+1)^2 + a*(2r+1) + b][p].
//
// Warp roles (192 threads): warp 0 issues TMA, warp 1 allocates TMEM and issues
// MMAs (one elected lane each), warps 2..5 are the epilogue; warp w reads TMEM
// lanes 32*(w%4) .. 32*(w%4)+31, i.e. tile pixels 32*(w%4) + lane.
//
// Every mbarrier wait is bounded (2 s); on a time-out the CTA raises the
// context's device error word, stops all roles, waits (bounded) for its TMA
// copies in flight, frees its TMEM and returns.  No TMA multicast is used.
#include <cuda.h>

#include "dc_internal.cuh"
#include "dc_sm100.cuh"

namespace {

using namespace dc::sm100;

constexpr int kTileM = 128;      // source pixels per CTA = MMA M = TMEM lanes
constexpr int kChunkN = 256;     // target pixels per chunk = MMA N (max)
constexpr int kThreads = 192;
constexpr int kMaxChunks = 128;
constexpr int kWinStride = 65;   // floats per pixel window row (64 taps + pad)
constexpr int kStStride = 33;    // floats per staged TMEM row (32 + pad)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAtomRowsBytes = 128;  // one 128-byte K atom per row

struct ChunkDesc {
    int level, q0, n, row;
};

struct TcParams {
    dc::Geom g;
    const int* ii;
    const int* jj;
    int max_frames;
    const float* coords;
    float* out;
    int* err;
    int atoms;        // 128-byte K atoms per operand row (C * 2 / 128)
    uint32_t ab_fmt;  // 0 fp16, 1 bf16
};

struct Layout {
    uint32_t a, b, stage_b, win, st, chunks, bars, misc, total;
};

__host__ __device__ inline Layout make_layout(int atoms) {
    Layout L;
    L.a = 0;
    L.b = L.a + atoms * kTileM * kAtomRowsBytes;
    L.stage_b = atoms * kChunkN * kAtomRowsBytes;
    L.win = L.b + 2 * L.stage_b;
    L.st = L.win + kTileM * kWinStride * 4;
    L.chunks = L.st + kTileM * kStStride * 4;
    L.bars = L.chunks + kMaxChunks * sizeof(ChunkDesc);
    L.misc = L.bars + 16 * 8;
    L.total = L.misc + 64;
    return L;
}

// misc words
enum { kMiscTmem = 0, kMiscAbort = 1, kMiscCount = 2, kMiscRange = 4 };  // range: 2 per level
// barrier slots
enum { kBarA = 0, kBarFull = 1, kBarEmpty = 3, kBarTFull = 5, kBarTEmpty = 7 };

__device__ __forceinline__ void raise_abort(volatile int* abort, int* err, int code) {
    *abort = 1;
    atomicExch(err, code);
}

template <int R>
__global__ void __launch_bounds__(kThreads, 1)
    corr_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b, TcParams P) {
    constexpr int D = 2 * R + 1, NW = 2 * R + 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const Layout Ly = make_layout(P.atoms);
    const dc::Geom& g = P.g;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.y, p0 = blockIdx.x * kTileM;
    const int hw = g.hw, nch = g.levels * D * D;
    float* out_e = P.out + (size_t)e * nch * hw;

    const int si = P.ii[e], sj = P.jj[e];
    if (!(si >= 0 && si < P.max_frames && sj >= 0 && sj < P.max_frames)) {
        for (int idx = threadIdx.x; idx < nch * kTileM; idx += kThreads) {
            const int p = p0 + (idx % kTileM);
            if (p < hw) out_e[(size_t)(idx / kTileM) * hw + p] = 0.0f;
        }
        return;
    }

    const uint32_t sA = smem_addr(base + Ly.a);
    const uint32_t sB = smem_addr(base + Ly.b);
    float* win_base = reinterpret_cast<float*>(base + Ly.win);
    float* st_base = reinterpret_cast<float*>(base + Ly.st);
    ChunkDesc* chunks = reinterpret_cast<ChunkDesc*>(base + Ly.chunks);
    const uint32_t bars = smem_addr(base + Ly.bars);
    int* misc = reinterpret_cast<int*>(base + Ly.misc);
    volatile int* abort = misc + kMiscAbort;
    auto bar = [&](int slot) { return bars + 8u * slot; };

    if (threadIdx.x == 0) {
        mbar_init(bar(kBarA), 1);
        for (int s = 0; s < 2; s++) {
            mbar_init(bar(kBarFull + s), 1);
            mbar_init(bar(kBarEmpty + s), 1);
            mbar_init(bar(kBarTFull + s), 1);
            mbar_init(bar(kBarTEmpty + s), 4);
        }
        misc[kMiscAbort] = 0;
        for (int l = 0; l < DC_MAX_LEVELS; l++) {
            misc[kMiscRange + 2 * l] = 0x7fffffff;
            misc[kMiscRange + 2 * l + 1] = -1;
        }
        fence_mbar_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(misc + kMiscTmem), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = (uint32_t)misc[kMiscTmem];

    // ---- 1. target-row range per level over this tile's windows
    const bool epi = warp >= 2;
    const int ti = 32 * (warp & 3) + lane;  // tile pixel (epilogue threads)
    const int p = p0 + ti;
    const bool pv = epi && p < hw;
    float cx = 0.0f, cy = 0.0f;
    if (pv) {
        cx = __ldg(P.coords + (size_t)e * 2 * hw + p);
        cy = __ldg(P.coords + (size_t)e * 2 * hw + hw + p);
        for (int l = 0; l < g.levels; l++) {
            const float y0 = cy * (1.0f / (float)(1 << l));
            const float x0 = cx * (1.0f / (float)(1 << l));
            const int by = (int)floorf(y0) - R, bx = (int)floorf(x0) - R;
            const int lo = max(by, 0), hi = min(by + NW - 1, g.H[l] - 1);
            const bool xin = bx + NW - 1 >= 0 && bx < g.W[l];
            if (lo <= hi && xin) {
                atomicMin(&misc[kMiscRange + 2 * l], lo);
                atomicMax(&misc[kMiscRange + 2 * l + 1], hi);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int n = 0;
        for (int l = 0; l < g.levels; l++) {
            const int ylo = misc[kMiscRange + 2 * l], yhi = misc[kMiscRange + 2 * l + 1];
            if (ylo > yhi) continue;
            const int qs = ylo * g.W[l], qe = (yhi + 1) * g.W[l];
            for (int q = qs; q < qe && n < kMaxChunks; q += kChunkN) {
                const int len = min(kChunkN, qe - q);
                ChunkDesc c;
                c.level = l;
                c.q0 = q;
                c.n = (len + 15) & ~15;
                c.row = (int)((long long)sj * g.frame_rows + g.row0[l] + q);
                chunks[n++] = c;
            }
        }
        misc[kMiscCount] = n;
    }
    __syncthreads();
    const int nchunks = misc[kMiscCount];

    if (warp == 0) {
        // ---- 2. TMA producer
        if (lane == 0) {
            const uint32_t a_bytes = P.atoms * kTileM * kAtomRowsBytes;
            const uint32_t b_bytes = Ly.stage_b;
            mbar_arrive_expect_tx(bar(kBarA), a_bytes);
            const int arow = (int)((long long)si * g.frame_rows + g.row0[0] + p0);
            for (int k = 0; k < P.atoms; k++)
                tma_load_2d(sA + k * kTileM * kAtomRowsBytes, &tmap_a, k * 64, arow, bar(kBarA));
            int issued = 0;
            for (int c = 0; c < nchunks; c++) {
                const int s = c & 1;
                if (c >= 2 && !mbar_wait(bar(kBarEmpty + s), ((c >> 1) - 1) & 1, abort)) {
                    raise_abort(abort, P.err, 1);
                    break;
                }
                mbar_arrive_expect_tx(bar(kBarFull + s), b_bytes);
                const ChunkDesc ch = chunks[c];
                for (int k = 0; k < P.atoms; k++)
                    tma_load_2d(sB + s * Ly.stage_b + k * kChunkN * kAtomRowsBytes, &tmap_b,
                                k * 64, ch.row, bar(kBarFull + s));
                issued = c + 1;
            }
            if (*abort) {
                // let this CTA's copies in flight land before the CTA exits
                mbar_wait(bar(kBarA), 0, nullptr);
                for (int c = max(0, issued - 2); c < issued; c++)
                    mbar_wait(bar(kBarFull + (c & 1)), (c >> 1) & 1, nullptr);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- 3. MMA issuer
        if (lane == 0) {
            if (!mbar_wait(bar(kBarA), 0, abort)) {
                raise_abort(abort, P.err, 2);
            } else {
                tc_fence_after();
                for (int c = 0; c < nchunks; c++) {
                    const int s = c & 1, u = c >> 1;
                    if (!mbar_wait(bar(kBarFull + s), u & 1, abort)) {
                        raise_abort(abort, P.err, 3);
                        break;
                    }
                    if (c >= 2 && !mbar_wait(bar(kBarTEmpty + s), (u - 1) & 1, abort)) {
                        raise_abort(abort, P.err, 4);
                        break;
                    }
                    tc_fence_after();
                    const ChunkDesc ch = chunks[c];
                    const uint32_t idesc = idesc_f16(P.ab_fmt, kTileM, ch.n);
                    const uint32_t d = tmem + (uint32_t)(s * kChunkN);
                    const int ksteps = P.atoms * 4;  // 16 elements (32 bytes) per MMA
                    for (int kk = 0; kk < ksteps; kk++) {
                        const int at = kk >> 2, wi = kk & 3;
                        const uint64_t ad = sdesc_sw128(sA + at * kTileM * kAtomRowsBytes + wi * 32);
                        const uint64_t bd = sdesc_sw128(sB + s * Ly.stage_b +
                                                        at * kChunkN * kAtomRowsBytes + wi * 32);
                        mma_f16(d, ad, bd, idesc, kk > 0 ? 1u : 0u);
                    }
                    mma_commit(bar(kBarEmpty + s));
                    mma_commit(bar(kBarTFull + s));
                }
            }
        }
        __syncwarp();
    } else {
        // ---- 4. epilogue
        float* win = win_base + ti * kWinStride;
        float* st = st_base + ti * kStStride;
        const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
        int c = 0;
        bool alive = true;
        for (int l = 0; l < g.levels && alive; l++) {
            const int Hl = g.H[l], Wl = g.W[l];
            const float scale = 1.0f / (float)(1 << l);
            const float x0 = cx * scale, y0 = cy * scale;
            const float fx = floorf(x0), fy = floorf(y0);
            const float dx = x0 - fx, dy = y0 - fy;
            const int bx = (int)fx - R, by = (int)fy - R;
            const int ylo = max(by, 0), yhi = min(by + NW - 1, Hl - 1);
            const int xlo = max(bx, 0), xhi = min(bx + NW - 1, Wl - 1);
            const bool any = pv && ylo <= yhi && xlo <= xhi;
            while (c < nchunks && chunks[c].level == l) {
                const int s = c & 1, u = c >> 1;
                int okw = 1;
                if (lane == 0) okw = mbar_wait(bar(kBarTFull + s), u & 1, abort) ? 1 : 0;
                okw = __shfl_sync(0xffffffffu, okw, 0);
                if (!okw) {
                    if (lane == 0) raise_abort(abort, P.err, 5);
                    alive = false;
                    break;
                }
                mbar_wait(bar(kBarTFull + s), u & 1, abort);
                tc_fence_after();
                const ChunkDesc ch = chunks[c];
                const int nsl = (ch.n + 31) >> 5;
                for (int t = 0; t < nsl; t++) {
                    const int qs = ch.q0 + 32 * t, qe = qs + 31;
                    bool need = false;
                    if (any) {
                        const int ya = qs / Wl, yb = qe / Wl;
                        need = ylo <= yb && yhi >= ya;
                    }
                    if (__any_sync(0xffffffffu, need)) {
                        float v[32];
                        tmem_ld32(tl + (uint32_t)(s * kChunkN + 32 * t), v);
                        if (need) {
#pragma unroll
                            for (int k = 0; k < 32; k++) st[k] = v[k];
                            for (int y = max(ylo, qs / Wl); y <= min(yhi, qe / Wl); y++) {
                                const int qrow = y * Wl;
                                const int qa = max(qrow + xlo, qs), qb = min(qrow + xhi, qe);
                                for (int q = qa; q <= qb; q++)
                                    win[(q - qrow - bx) * 8 + (y - by)] = g.alpha * st[q - qs];
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(kBarTEmpty + s));
                c++;
            }
            if (!alive) break;
            if (pv) {
                bool vx[NW], vy[NW];
#pragma unroll
                for (int k = 0; k < NW; k++) {
                    vx[k] = (unsigned)(bx + k) < (unsigned)Wl;
                    vy[k] = (unsigned)(by + k) < (unsigned)Hl;
                }
                const float ux = 1.0f - dx, uy = 1.0f - dy;
                float* ol = out_e + (size_t)(l * D * D) * hw + p;
#pragma unroll
                for (int a = 0; a < D; a++)
#pragma unroll
                    for (int b = 0; b < D; b++) {
                        float acc = 0.0f;
                        acc = dc::bilinear_tap(acc, win[a * 8 + b], vx[a] && vy[b], ux, uy);
                        acc = dc::bilinear_tap(acc, win[a * 8 + b + 1], vx[a] && vy[b + 1], ux, dy);
                        acc = dc::bilinear_tap(acc, win[(a + 1) * 8 + b], vx[a + 1] && vy[b], dx, uy);
                        acc = dc::bilinear_tap(acc, win[(a + 1) * 8 + b + 1], vx[a + 1] && vy[b + 1], dx, dy);
                        __stcs(ol + (size_t)(a * D + b) * hw, acc);
                    }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

}  // namespace

bool dc_tc_supported(const dc_ctx* ctx) {
    const int p = ctx->cfg.precision;
    return (p == DC_PREC_FP16 || p == DC_PREC_BF16) &&
           (ctx->cfg.channels == 64 || ctx->cfg.channels == 128);
}

// Tensor maps over the store, [max_frames * frame_rows][C] 16-bit elements:
// A tiles of 128 rows and B chunks of 256 rows, 64 elements (128 bytes) wide,
// 128-byte swizzle (the canonical K-major operand layout of tcgen05).
int dc_tc_prepare(dc_ctx* ctx) {
    EncodeTiledFn enc = get_encode();
    if (!enc) return dc_fail(ctx, DC_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const CUtensorMapDataType dt = ctx->cfg.precision == DC_PREC_BF16
                                       ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    cuuint64_t dims[2] = {(cuuint64_t)ctx->cfg.channels,
                          (cuuint64_t)ctx->cfg.max_frames * ctx->frame_rows};
    cuuint64_t strides[1] = {(cuuint64_t)ctx->cfg.channels * 2};
    cuuint32_t estr[2] = {1, 1};
    cuuint32_t box_a[2] = {64, (cuuint32_t)kTileM};
    cuuint32_t box_b[2] = {64, (cuuint32_t)kChunkN};
    CUresult r1 = enc(reinterpret_cast<CUtensorMap*>(ctx->tmap_a), dt, 2, ctx->store, dims,
                      strides, box_a, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CUresult r2 = enc(reinterpret_cast<CUtensorMap*>(ctx->tmap_b), dt, 2, ctx->store, dims,
                      strides, box_b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS)
        return dc_fail(ctx, DC_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    ctx->tc_ready = true;
    return DC_OK;
}

int dc_launch_tc(dc_ctx* ctx, const int* ii, const int* jj, int M, const float* coords,
                 float* out, cudaStream_t s) {
    if (!ctx->tc_ready) return dc_fail(ctx, DC_ERR_NOT_READY, "tensor maps not prepared");
    TcParams P;
    P.g = dc::geom_of(ctx);
    P.ii = ii;
    P.jj = jj;
    P.max_frames = ctx->cfg.max_frames;
    P.coords = coords;
    P.out = out;
    P.err = ctx->dev_err;
    P.atoms = ctx->cfg.channels * 2 / 128;
    P.ab_fmt = ctx->cfg.precision == DC_PREC_BF16 ? 1u : 0u;
    const Layout Ly = make_layout(P.atoms);
    const size_t smem = Ly.total + 1024;
    dim3 grid((ctx->hw + kTileM - 1) / kTileM, M);
    const CUtensorMap* ta = reinterpret_cast<const CUtensorMap*>(ctx->tmap_a);
    const CUtensorMap* tb = reinterpret_cast<const CUtensorMap*>(ctx->tmap_b);
#define DC_TC_LAUNCH(RR)                                                                   \
    do {                                                                                   \
        auto k = corr_tc_kernel<RR>;                                                       \
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);   \
        k<<<grid, kThreads, smem, s>>>(*ta, *tb, P);                                       \
    } while (0)
    switch (ctx->cfg.radius) {
        case 0: DC_TC_LAUNCH(0); break;
        case 1: DC_TC_LAUNCH(1); break;
        case 2: DC_TC_LAUNCH(2); break;
        default: DC_TC_LAUNCH(3); break;
    }
#undef DC_TC_LAUNCH
    return dc_check_launch(ctx, "corr_tc_kernel");
}

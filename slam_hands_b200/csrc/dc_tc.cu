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
//      K-major operand) through shared memory with TMA in row-aligned chunks of
//      at most 128 target pixels, double-buffered;
//   3. computes each 128 x n x C correlation chunk with tcgen05.mma (kind::f16,
//      fp16 or bf16 operands, fp32 accumulation in TMEM, four accumulators so the
//      epilogue of chunk c overlaps the MMAs of the next chunks);
//   4. reads back only the TMEM columns that hold some pixel's window taps
//      (tcgen05.ld), stages the 16-byte groups a pixel needs in shared memory,
//      picks its taps into its window, and after the last chunk of a level forms
//      the (2r+1)^2 bilinear outputs in the reference's rounding order
//      (main.cu:1196-1213), stored as coalesced 128-byte rows of
//      out[e][l*(2r+1)^2 + a*(2r+1) + b][p].
//
// Warp roles (320 threads): warp 0 issues TMA, warp 1 allocates TMEM and issues
// MMAs (one elected lane each), warps 2..9 are the epilogue.  Warp w reads TMEM
// lanes 32*(w%4) .. 32*(w%4)+31, i.e. tile pixels 32*(w%4) + lane; the two warps
// of a lane quarter take the two 64-column halves of a chunk and split the
// outputs.
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
constexpr int kChunkN = 256;     // max target pixels per chunk = MMA N
constexpr int kSubCols = 32;     // chunk columns per epilogue warp
constexpr int kStagesB = 2;      // shared-memory stages of target rows
constexpr int kAcc = 2;          // TMEM accumulators (kAcc * kChunkN = 512 columns)
constexpr int kSubWarps = 4;     // epilogue warps per TMEM lane quarter
constexpr int kPasses = kChunkN / (kSubWarps * 32);  // 32-column passes per warp and chunk
constexpr int kEpiWarps = 4 * kSubWarps;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kWinStride = 65;   // floats per pixel window row (64 taps + pad)
constexpr int kStStride = 12;   // floats per staging row: 3 16-byte groups (bank-conflict free)
constexpr uint32_t kTmemCols = kAcc * kChunkN;
constexpr uint32_t kRowBytes = 128;  // one 128-byte K atom per operand row

// A chunk is `nrows` consecutive target rows of one level, each the segment
// [x0, x0 + seg) of the row (seg = W when whole rows fit, else a row is split).
struct ChunkDesc {
    int n, row;            // MMA N (multiple of 16), store row of the first pixel
    int y0, x0, seg, cols; // level coordinates of chunk column 0, segment, columns
};

// Per-level chunk schedule of one tile: chunks first .. first+count-1 cover the
// target rows ylo..yhi of the level, rows_per whole rows per chunk, or for rows
// wider than a chunk, segs segments of seg_max pixels per row.
struct LevelSched {
    int first, count, ylo, yhi, rows_per, seg_max, segs, W;
};

__device__ __forceinline__ ChunkDesc make_chunk(const LevelSched& L, int idx,
                                                long long row_base) {
    ChunkDesc c;
    int r = idx, sg = 0;
    if (L.segs > 1) {
        r = idx / L.segs;
        sg = idx - r * L.segs;
    }
    c.y0 = L.ylo + r * L.rows_per;
    c.x0 = sg * L.seg_max;
    c.seg = min(L.seg_max, L.W - c.x0);
    c.cols = min(L.rows_per, L.yhi - c.y0 + 1) * c.seg;
    c.n = (c.cols + 15) & ~15;
    c.row = (int)(row_base + (long long)c.y0 * L.W + c.x0);
    return c;
}

// floor(v / d) for 0 <= v < 2^12 and 1 <= d <= 2^12 from d's reciprocal: the
// quotient of v + 0.5 is at least 0.5 / d away from an integer, far above the
// rounding error of the product.
__device__ __forceinline__ int div_small(int v, float inv_d) {
    return (int)(((float)v + 0.5f) * inv_d);
}

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
    int M;            // edges
};

struct TileInfo {
    int e, p0, si, sj, n, valid, pad0, pad1;
};

struct Layout {
    uint32_t a, b, stage_b, win, st, sched, tinfo, coords, bars, misc, total;
};

__host__ __device__ constexpr Layout make_layout(int atoms) {
    Layout L{};
    L.a = 0;
    L.b = L.a + atoms * kTileM * kRowBytes;
    L.stage_b = atoms * kChunkN * kRowBytes;
    L.win = L.b + kStagesB * L.stage_b;
    L.st = L.win + kTileM * kWinStride * 4;
    L.sched = L.st;                                          // [2][levels] LevelSched
    L.tinfo = L.sched + 2 * DC_MAX_LEVELS * sizeof(LevelSched);
    L.coords = L.tinfo + 2 * sizeof(TileInfo);              // [2][2][128] floats
    L.bars = L.coords + 2 * 2 * kTileM * 4;
    L.misc = L.bars + 24 * 8;
    L.total = L.misc + 64;
    return L;
}
static_assert(make_layout(2).total + 1024 <= 227 * 1024, "shared memory budget");

// misc words
enum { kMiscTmem = 0, kMiscAbort = 1 };
// barrier slots: A tile full/empty, B stages full/empty, TMEM accumulators
// full/empty, per-tile schedule full/empty (double-buffered by tile parity)
enum { kBarAFull = 0, kBarAEmpty = 1, kBarFull = 2, kBarEmpty = kBarFull + kStagesB,
       kBarTFull = kBarEmpty + kStagesB, kBarTEmpty = kBarTFull + kAcc,
       kBarSFull = kBarTEmpty + kAcc, kBarSEmpty = kBarSFull + 2 };
static_assert(kBarSEmpty + 2 <= 24, "barrier slots");

__device__ __forceinline__ void raise_abort(volatile int* abort, int* err, int code) {
    *abort = 1;
    atomicExch(err, code);
}

// Optional phase timers (build with -DDC_TC_PROFILE; compiled out otherwise):
// per CTA, cycles spent in each role's waits and in the epilogue phases.
#ifdef DC_TC_PROFILE
__device__ unsigned long long g_tc_prof[8192 * 16];
#define DC_PROF_NOW() clock64()
#define DC_PROF_STORE(slot, v)                                                    \
    do {                                                                          \
        const int cta_ = blockIdx.x;                                              \
        if (cta_ < 8192) g_tc_prof[cta_ * 16 + (slot)] = (unsigned long long)(v); \
    } while (0)
#else
#define DC_PROF_NOW() 0ll
#define DC_PROF_STORE(slot, v) \
    do {                       \
    } while (0)
#endif

// Named barrier of the kSubWarps epilogue warps that share a TMEM lane quarter.
__device__ __forceinline__ void quarter_sync(int quarter) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + quarter), "r"(32 * kSubWarps) : "memory");
}

// All lanes of a warp wait for one barrier phase: lane 0 polls (bounded), the
// others then observe the completed phase.  Returns false on a time-out.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                          int lane) {
    int ok = 1;
    if (lane == 0) ok = mbar_wait(bar, parity, abort) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) mbar_wait(bar, parity, abort);
    return ok != 0;
}

// Persistent: CTA b handles tiles b, b + gridDim.x, ...; tile t = (edge t / tpe,
// source pixels 128 * (t % tpe) ..).  The producer warp also prepares each
// tile's coordinates and chunk schedule one tile ahead, so a tile's set-up and
// its last level's bilinear step overlap the neighbouring tiles' MMAs.
template <int R>
__global__ void __launch_bounds__(kThreads, 1)
    corr_tc_kernel(const __grid_constant__ CUtensorMap tmap, TcParams P) {
    constexpr int D = 2 * R + 1, NW = 2 * R + 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr Layout Ly2 = make_layout(2);
    const Layout Ly = P.atoms == 2 ? Ly2 : make_layout(P.atoms);
    const dc::Geom& g = P.g;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hw = g.hw, nch = g.levels * D * D;
    const int tpe = (hw + kTileM - 1) / kTileM;  // tiles per edge
    const int ntiles = tpe * P.M;
    const long long t_start = DC_PROF_NOW();
    (void)t_start;

    const uint32_t sA = smem_addr(base + Ly.a);
    const uint32_t sB = smem_addr(base + Ly.b);
    float* win_base = reinterpret_cast<float*>(base + Ly.win);
    LevelSched* sched_base = reinterpret_cast<LevelSched*>(base + Ly.sched);
    TileInfo* tinfo = reinterpret_cast<TileInfo*>(base + Ly.tinfo);
    float* scoords = reinterpret_cast<float*>(base + Ly.coords);
    const uint32_t bars = smem_addr(base + Ly.bars);
    int* misc = reinterpret_cast<int*>(base + Ly.misc);
    volatile int* abort = misc + kMiscAbort;
    auto bar = [&](int slot) { return bars + 8u * slot; };

    if (threadIdx.x == 0) {
        mbar_init(bar(kBarAFull), 1);
        mbar_init(bar(kBarAEmpty), 1);
        for (int s = 0; s < kStagesB; s++) {
            mbar_init(bar(kBarFull + s), 1);
            mbar_init(bar(kBarEmpty + s), 1);
        }
        for (int a = 0; a < kAcc; a++) {
            mbar_init(bar(kBarTFull + a), 1);
            mbar_init(bar(kBarTEmpty + a), kEpiWarps);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(bar(kBarSFull + b), 1);
            mbar_init(bar(kBarSEmpty + b), kEpiWarps + 1);
        }
        misc[kMiscAbort] = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmap);
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(misc + kMiscTmem), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = (uint32_t)misc[kMiscTmem];
    long long w_a = 0, w_b = 0, w_c = 0;  // phase cycles (profiling builds)

    if (warp == 0) {
        // ---- producer: per tile, coordinates + chunk schedule, then the source
        //      tile and the target-row chunks through TMA
        int gc = 0, na = 0, i = 0;
        int a_issued = 0, last_gc = 0;
        for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x, i++) {
            const int tb = i & 1;
            if (i >= 2 && !warp_wait(bar(kBarSEmpty + tb), ((i >> 1) - 1) & 1, abort, lane)) {
                if (lane == 0) raise_abort(abort, P.err, 1);
                break;
            }
            const int e = t / tpe, p0 = (t - e * tpe) * kTileM;
            const int si = P.ii[e], sj = P.jj[e];
            const bool valid = si >= 0 && si < P.max_frames && sj >= 0 && sj < P.max_frames;
            float* sc = scoords + tb * 2 * kTileM;
            int lo[DC_MAX_LEVELS], hi[DC_MAX_LEVELS];
#pragma unroll
            for (int l = 0; l < DC_MAX_LEVELS; l++) {
                lo[l] = 0x7fffffff;
                hi[l] = -1;
            }
#pragma unroll
            for (int k = 0; k < kTileM / 32; k++) {
                const int q = lane + 32 * k, p = p0 + q;
                float cx = 0.0f, cy = 0.0f;
                if (p < hw) {
                    cx = __ldg(P.coords + (size_t)e * 2 * hw + p);
                    cy = __ldg(P.coords + (size_t)e * 2 * hw + hw + p);
                }
                sc[q] = cx;
                sc[kTileM + q] = cy;
                if (!(valid && p < hw)) continue;
#pragma unroll
                for (int l = 0; l < DC_MAX_LEVELS; l++) {
                    if (l >= g.levels) break;
                    const float s = 1.0f / (float)(1 << l);
                    const int by = (int)floorf(cy * s) - R, bx = (int)floorf(cx * s) - R;
                    const int a0 = max(by, 0), a1 = min(by + NW - 1, g.H[l] - 1);
                    if (a0 <= a1 && bx + NW - 1 >= 0 && bx < g.W[l]) {
                        lo[l] = min(lo[l], a0);
                        hi[l] = max(hi[l], a1);
                    }
                }
            }
            int n = 0;
#pragma unroll
            for (int l = 0; l < DC_MAX_LEVELS; l++) {
                const int ylo = __reduce_min_sync(0xffffffffu, lo[l]);
                const int yhi = __reduce_max_sync(0xffffffffu, hi[l]);
                LevelSched L;
                L.first = n;
                L.count = 0;
                L.ylo = ylo;
                L.yhi = yhi;
                L.W = max(g.W[l], 1);
                L.rows_per = L.W <= kChunkN ? kChunkN / L.W : 1;
                L.seg_max = L.W <= kChunkN ? L.W : kChunkN;
                L.segs = (L.W + L.seg_max - 1) / L.seg_max;
                if (l < g.levels && ylo <= yhi)
                    L.count = (yhi - ylo + L.rows_per) / L.rows_per * L.segs;
                n += L.count;
                if (lane == 0) sched_base[tb * DC_MAX_LEVELS + l] = L;
            }
            if (lane == 0) {
                TileInfo ti;
                ti.e = e;
                ti.p0 = p0;
                ti.si = si;
                ti.sj = sj;
                ti.n = n;
                ti.valid = valid;
                ti.pad0 = ti.pad1 = 0;
                tinfo[tb] = ti;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarSFull + tb));  // release: schedule, coords
            if (n == 0) continue;
            if (lane == 0) {
                // the single source-tile buffer: wait until the MMAs of the previous
                // tile that used it are done
                if (na >= 1 && !mbar_wait(bar(kBarAEmpty), (na - 1) & 1, abort)) {
                    raise_abort(abort, P.err, 2);
                } else {
                    mbar_arrive_expect_tx(bar(kBarAFull), P.atoms * kTileM * kRowBytes);
                    const int arow = (int)((long long)si * g.frame_rows + g.row0[0] + p0);
                    for (int k = 0; k < P.atoms; k++)
                        tma_load_2d(sA + k * kTileM * kRowBytes, &tmap, k * 64, arow,
                                    bar(kBarAFull));
                    a_issued = 1;
                    const LevelSched* sch = sched_base + tb * DC_MAX_LEVELS;
                    int lv = 0;
                    for (int c = 0; c < n; c++, gc++) {
                        while (c >= sch[lv].first + sch[lv].count) lv++;
                        const int s = gc % kStagesB;
                        const long long t0 = DC_PROF_NOW();
                        if (gc >= kStagesB &&
                            !mbar_wait(bar(kBarEmpty + s), ((gc / kStagesB) - 1) & 1, abort)) {
                            raise_abort(abort, P.err, 3);
                            break;
                        }
                        w_a += DC_PROF_NOW() - t0;
                        mbar_arrive_expect_tx(bar(kBarFull + s), Ly.stage_b);
                        const int row = make_chunk(sch[lv], c - sch[lv].first,
                                                   (long long)sj * g.frame_rows + g.row0[lv]).row;
                        for (int k = 0; k < P.atoms; k++)
                            for (int h = 0; h < kChunkN / kTileM; h++)  // 128-row boxes
                                tma_load_2d(sB + s * Ly.stage_b + k * kChunkN * kRowBytes +
                                                h * kTileM * kRowBytes,
                                            &tmap, k * 64, row + h * kTileM, bar(kBarFull + s));
                        last_gc = gc + 1;
                    }
                }
            }
            na++;
            __syncwarp();
        }
        if (lane == 0) {
            DC_PROF_STORE(4, w_a);
            if (*abort) {
                // let this CTA's copies in flight land before the CTA exits
                if (a_issued) mbar_wait(bar(kBarAFull), (na - 1) & 1, nullptr);
                for (int c = max(0, last_gc - kStagesB); c < last_gc; c++)
                    mbar_wait(bar(kBarFull + c % kStagesB), (c / kStagesB) & 1, nullptr);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer
        int gc = 0, na = 0, i = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, i++) {
            const int tb = i & 1;
            if (!warp_wait(bar(kBarSFull + tb), (i >> 1) & 1, abort, lane)) {
                if (lane == 0) raise_abort(abort, P.err, 4);
                break;
            }
            const TileInfo ti = tinfo[tb];
            const LevelSched* sch = sched_base + tb * DC_MAX_LEVELS;
            bool ok = true;
            if (lane == 0 && ti.n > 0) {
                if (!mbar_wait(bar(kBarAFull), na & 1, abort)) {
                    raise_abort(abort, P.err, 5);
                    ok = false;
                } else {
                    tc_fence_after();
                    const int ksteps = P.atoms * 4;  // 16 elements (32 bytes) per MMA
                    int lv = 0;
                    for (int c = 0; c < ti.n; c++, gc++) {
                        while (c >= sch[lv].first + sch[lv].count) lv++;
                        const int s = gc % kStagesB, a = gc % kAcc;
                        const long long t0 = DC_PROF_NOW();
                        if (!mbar_wait(bar(kBarFull + s), (gc / kStagesB) & 1, abort)) {
                            raise_abort(abort, P.err, 6);
                            ok = false;
                            break;
                        }
                        const long long t1 = DC_PROF_NOW();
                        w_a += t1 - t0;
                        if (gc >= kAcc &&
                            !mbar_wait(bar(kBarTEmpty + a), ((gc / kAcc) - 1) & 1, abort)) {
                            raise_abort(abort, P.err, 7);
                            ok = false;
                            break;
                        }
                        w_b += DC_PROF_NOW() - t1;
                        tc_fence_after();
                        const int nn = make_chunk(sch[lv], c - sch[lv].first, 0).n;
                        const uint32_t idesc = idesc_f16(P.ab_fmt, kTileM, nn);
                        const uint32_t d = tmem + (uint32_t)(a * kChunkN);
                        for (int kk = 0; kk < ksteps; kk++) {
                            const int at = kk >> 2, wi = kk & 3;
                            const uint64_t ad = sdesc_sw128(sA + at * kTileM * kRowBytes + wi * 32);
                            const uint64_t bd = sdesc_sw128(sB + s * Ly.stage_b +
                                                            at * kChunkN * kRowBytes + wi * 32);
                            mma_f16(d, ad, bd, idesc, kk > 0 ? 1u : 0u);
                        }
                        mma_commit(bar(kBarEmpty + s));
                        mma_commit(bar(kBarTFull + a));
                    }
                    mma_commit(bar(kBarAEmpty));  // the source tile may be replaced
                }
            }
            if (ti.n > 0) na++;
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (lane == 0) mbar_arrive(bar(kBarSEmpty + tb));
            if (!ok) break;
        }
        if (lane == 0) {
            DC_PROF_STORE(2, w_a);
            DC_PROF_STORE(3, w_b);
            DC_PROF_STORE(8, gc);
            DC_PROF_STORE(9, i);
        }
        __syncwarp();
    } else {
        // ---- epilogue: the kSubWarps warps of a TMEM lane quarter take the
        //      32-column passes of each chunk and split the outputs
        const int quarter = warp & 3;       // TMEM lane quarter of this warp
        const int sub = (warp - 2) >> 2;    // which columns of a chunk (0..kSubWarps-1)
        const int ti_px = 32 * quarter + lane;
        float* win = win_base + ti_px * kWinStride;
        const uint32_t tl = tmem + ((uint32_t)(32 * quarter) << 16);
        const int cwarp = kSubCols * kPasses * sub;  // first chunk column of this warp
        int gc = 0, i = 0;
        bool alive = true;
        for (int t = blockIdx.x; t < ntiles && alive; t += gridDim.x, i++) {
            const int tb = i & 1;
            const long long t0s = DC_PROF_NOW();
            if (!warp_wait(bar(kBarSFull + tb), (i >> 1) & 1, abort, lane)) {
                if (lane == 0) raise_abort(abort, P.err, 8);
                break;
            }
            w_a += DC_PROF_NOW() - t0s;
            const TileInfo tinf = tinfo[tb];
            const LevelSched* sch = sched_base + tb * DC_MAX_LEVELS;
            const int p = tinf.p0 + ti_px;
            const bool pv = p < hw;
            const bool valid = tinf.valid != 0;
            const float cx = scoords[tb * 2 * kTileM + ti_px];
            const float cy = scoords[tb * 2 * kTileM + kTileM + ti_px];
            float* out_e = P.out + (size_t)tinf.e * nch * hw;
            int cend = 0;
            for (int l = 0; l < g.levels && alive; l++) {
                const int Hl = g.H[l], Wl = g.W[l];
                const float scale = 1.0f / (float)(1 << l);
                const float x0 = cx * scale, y0 = cy * scale;
                const float fx = floorf(x0), fy = floorf(y0);
                const float dx = x0 - fx, dy = y0 - fy;
                const int bx = (int)fx - R, by = (int)fy - R;
                const int ylo = max(by, 0), yhi = min(by + NW - 1, Hl - 1);
                const int xlo = max(bx, 0), xhi = min(bx + NW - 1, Wl - 1);
                const bool any = valid && pv && ylo <= yhi && xlo <= xhi;
                const LevelSched Ls = sch[l];
                const float inv_seg_max = 1.0f / (float)Ls.seg_max;
                cend += Ls.count;
                for (int c = 0; c < Ls.count; c++, gc++) {
                    const int a = gc % kAcc;
                    const long long t0 = DC_PROF_NOW();
                    if (!warp_wait(bar(kBarTFull + a), (gc / kAcc) & 1, abort, lane)) {
                        if (lane == 0) raise_abort(abort, P.err, 9);
                        alive = false;
                        break;
                    }
                    tc_fence_after();
                    const long long t1 = DC_PROF_NOW();
                    w_a += t1 - t0;
                    const ChunkDesc ch = make_chunk(Ls, c, 0);
                    const float inv_seg =
                        ch.seg == Ls.seg_max ? inv_seg_max : 1.0f / (float)ch.seg;
#pragma unroll
                    for (int pass = 0; pass < kPasses; pass++) {
                        const int cb = cwarp + kSubCols * pass;
                        if (cb >= ch.cols) continue;
                        const int rlo = div_small(cb, inv_seg);
                        const int rhi = div_small(min(ch.cols - 1, cb + kSubCols - 1), inv_seg);
                        // window rows of this pixel inside this pass's chunk rows; tap
                        // (x, y) sits at staged column (y - y0) * seg + (x - x0) - cb
                        const int ya = max(ylo, ch.y0 + rlo);
                        const int yb = min(yhi, ch.y0 + rhi);
                        const int xa = max(xlo, ch.x0), xb = min(xhi, ch.x0 + ch.seg - 1);
                        bool need = any && ya <= yb && xa <= xb;
#if defined(DC_TC_EXP) && DC_TC_EXP == 2
                        need = false;
#endif
                        if (!__any_sync(0xffffffffu, need)) continue;
                        float v[kSubCols];
                        tmem_ld32(tl + (uint32_t)(a * kChunkN + cb), v);
#if defined(DC_TC_EXP) && DC_TC_EXP == 1
                        if (v[5] != 1234.5f) continue;
#endif
                        if (!need) continue;
                        const int kofs = -ch.x0 - cb;
                        const int ia = xa - bx, ib = xb - bx;  // valid tap range
                        for (int y = ya; y <= yb; y++) {
                            const int k0 = (y - ch.y0) * ch.seg + bx + kofs;
                            const int lo = max(ia, -k0), hi = min(ib, kSubCols - 1 - k0);
                            if (lo > hi) continue;
                            const unsigned span = (unsigned)(hi - lo);
                            // tap q sits at column k0 + q; the tap whose column is
                            // congruent to r mod 8 is in register 8 * (column >> 3) + r,
                            // so each of the 8 residues needs only a 4-way select
                            float* wcol = win + (y - by);
#pragma unroll
                            for (int r = 0; r < 8; r++) {
                                const int q = (r - k0) & 7;
                                const int kk = (k0 + q) >> 3;
                                const float val = (kk & 2) ? ((kk & 1) ? v[24 + r] : v[16 + r])
                                                           : ((kk & 1) ? v[8 + r] : v[r]);
                                if ((unsigned)(q - lo) <= span) wcol[q * 8] = g.alpha * val;
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar(kBarTEmpty + a));
                    w_b += DC_PROF_NOW() - t1;
                }
                if (!alive) break;
                const long long t2 = DC_PROF_NOW();
                quarter_sync(quarter);  // all passes have written this level's windows
                if (pv) {
                    bool vy[NW];
#pragma unroll
                    for (int k = 0; k < NW; k++)
                        vy[k] = any && (unsigned)(by + k) < (unsigned)Hl;
                    const float ux = 1.0f - dx, uy = 1.0f - dy;
                    float* ol = out_e + (size_t)(l * D * D) * hw + p;
                    // the quarter's warps split the output columns a (2, 2, 2, 1 at R = 3)
                    constexpr int AW = (D + kSubWarps - 1) / kSubWarps;
                    const int a0 = sub * AW;
                    // taps of columns a0 .. a0 + AW, premultiplied by the x weights;
                    // taps outside the level read as +0, which leaves every fmaf
                    // below unchanged, as skipping them does in the reference
                    float pu[AW + 1][NW], pd[AW + 1][NW];
#pragma unroll
                    for (int ii = 0; ii <= AW; ii++) {
                        const int ix = a0 + ii;
                        const bool vx = ix < NW && (unsigned)(bx + ix) < (unsigned)Wl;
#pragma unroll
                        for (int j = 0; j < NW; j++) {
                            const float tt = (vx && vy[j]) ? win[ix * 8 + j] : 0.0f;
                            pu[ii][j] = tt * ux;
                            pd[ii][j] = tt * dx;
                        }
                    }
#pragma unroll
                    for (int ai = 0; ai < AW; ai++) {
                        const int aa = a0 + ai;
                        if (aa >= D) break;
#pragma unroll
                        for (int b = 0; b < D; b++) {
                            // reference order: taps (a,b), (a,b+1), (a+1,b), (a+1,b+1)
                            float acc = fmaf(pu[ai][b], uy, 0.0f);
                            acc = fmaf(pu[ai][b + 1], dy, acc);
                            acc = fmaf(pd[ai + 1][b], uy, acc);
                            acc = fmaf(pd[ai + 1][b + 1], dy, acc);
                            __stcs(ol + (size_t)(aa * D + b) * hw, acc);
                        }
                    }
                }
                quarter_sync(quarter);  // all are done reading before the next level
                w_c += DC_PROF_NOW() - t2;
            }
            (void)cend;
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarSEmpty + tb));
        }
        if (lane == 0 && warp == 2) {
            DC_PROF_STORE(5, w_a);
            DC_PROF_STORE(6, w_b);
            DC_PROF_STORE(7, w_c);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (threadIdx.x == 0) DC_PROF_STORE(0, DC_PROF_NOW() - t_start);
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

#ifdef DC_TC_PROFILE
extern "C" int dc_tc_profile_read(unsigned long long* host, int n) {
    return (int)cudaMemcpyFromSymbol(host, g_tc_prof, sizeof(unsigned long long) * n);
}
#endif

bool dc_tc_supported(const dc_ctx* ctx) {
    const int p = ctx->cfg.precision;
    return (p == DC_PREC_FP16 || p == DC_PREC_BF16) &&
           (ctx->cfg.channels == 64 || ctx->cfg.channels == 128);
}

// Tensor map over the store, [max_frames * frame_rows][C] 16-bit elements, with
// boxes of 128 rows x 64 elements (128 bytes) and 128-byte swizzle: the
// canonical K-major operand layout of tcgen05, for A tiles and B chunks alike.
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
    static_assert(kChunkN % kTileM == 0, "B chunks are whole 128-row boxes");
    cuuint32_t box[2] = {64, (cuuint32_t)kTileM};
    CUresult r1 = enc(reinterpret_cast<CUtensorMap*>(ctx->tmap_a), dt, 2, ctx->store, dims,
                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r1 != CUDA_SUCCESS)
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
    P.M = M;
    const int ntiles = (ctx->hw + kTileM - 1) / kTileM * M;
    dim3 grid(ntiles < ctx->num_sms ? ntiles : ctx->num_sms);
    const CUtensorMap* ta = reinterpret_cast<const CUtensorMap*>(ctx->tmap_a);
#define DC_TC_LAUNCH(RR)                                                                   \
    do {                                                                                   \
        auto k = corr_tc_kernel<RR>;                                                       \
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);   \
        k<<<grid, kThreads, smem, s>>>(*ta, P);                                       \
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

// dc_tc.cu -- fused build + pyramid + lookup on the 5th-generation tensor cores.
//
// Drop-in for CudaDroid::batch_build_and_sample_correlation
// (cuda_slam/main.cu:1555-1613) that never writes a volume.  For one edge e and
// one tile of 128 source pixels p, the lookup needs, per level l, the volume
// values V_l[p][q] = alpha * <f_ii[:, p], P_l f_jj[:, q]> at the (2r+2)^2 taps
// around each pixel's scaled coordinate.  Per tile:
//   1. the producer warp reduces, over the tile's 128 pixels (coordinates
//      loaded one tile ahead), the range of target rows (and, for rows wider
//      than 256 pixels, of row segments) any window of level l touches;
//   2. the producer streams those rows of the pooled target map P_l f_jj
//      (pixel-major store, K-major operand) into shared memory: one 4-D TMA box
//      per 64-channel K atom holds `br` whole rows of `wbox` pixels (rows padded
//      to a multiple of 8 pixels, out-of-image pixels read as zeros), at most 256
//      targets -- few, large boxes, because a TMA box costs a fixed few hundred
//      cycles whatever its size;
//   3. one thread computes each 128 x N x C chunk with tcgen05.mma (kind::f16,
//      fp16 or bf16 operands, fp32 accumulation in TMEM, two accumulators so the
//      epilogue of one chunk overlaps the MMAs of the next);
//   4. the epilogue drains each chunk in 64-column loads (tcgen05.ld) of eight
//      8-column strips, every strip 8 consecutive target pixels of one row
//      starting at a multiple of 8.  A window of 8 columns starting at bx
//      touches only strips bx/8 and bx/8 + 1 of each of its rows (a 32-bit mask
//      over the chunk's strips), so a lane copies a strip it needs into slot 0
//      or 1 of its window row with two 16-byte stores -- no per-tap selection;
//   5. after the last chunk of a level, forms the (2r+1)^2 bilinear outputs
//      with the reference's weights (main.cu:1196-1213), evaluated separably,
//      reading window column x at slot column (bx mod 8) + x, and stores them as
//      out[e][l*(2r+1)^2 + a*(2r+1) + b][p] (consecutive pixels per warp).
//
// A tile is 128 consecutive source pixels, or, in the window-row tile order
// (dc_set_tile_order), 128 positions of a per-edge permutation that groups
// pixels by the row of their level-0 window: tile_order_kernel sorts each
// edge first, the producer then gathers the source rows with tile::gather4,
// the epilogue writes outputs at the tile position, and unpermute_rows_kernel
// moves them to pixel order after the call.
//
// Warp roles (320 threads): warp 0 schedules tiles and issues TMA, warp 1
// allocates TMEM and issues MMAs (one elected lane each), warps 2..9 are the
// epilogue.  Warp w reads TMEM lanes 32*(w%4) .. 32*(w%4)+31, i.e. tile pixels
// 32*(w%4) + lane; the two warps of a lane quarter take 128 columns of every
// chunk each (two 64-column loads) and split the bilinear outputs by column.
//
// Every mbarrier wait is bounded (2 s); on a time-out the CTA raises the
// context's device error word, stops all roles, waits (bounded) for its TMA
// copies in flight, frees its TMEM and returns.  No TMA multicast is used.
#include <cuda.h>

#include <atomic>
#include <cstring>

#include "dc_internal.cuh"
#include "dc_sm100.cuh"

namespace {

using namespace dc::sm100;

constexpr int kTileM = 128;      // source pixels per CTA = MMA M = TMEM lanes
#ifndef DC_TC_CHUNKN
#define DC_TC_CHUNKN 256
#endif
#ifndef DC_TC_STAGES_B
#define DC_TC_STAGES_B 2
#endif
constexpr int kChunkN = DC_TC_CHUNKN;  // max targets per chunk = MMA N
constexpr int kStrip = 8;        // target pixels per strip
constexpr int kChunkStrips = kChunkN / kStrip;  // 32 strips per chunk
constexpr int kStagesB = DC_TC_STAGES_B;  // shared-memory stages of target rows
constexpr int kAccCols = kChunkN;         // TMEM columns per accumulator
constexpr int kAcc = 512 / kAccCols;      // TMEM accumulators
#ifndef DC_TC_SUBWARPS
#define DC_TC_SUBWARPS 2
#endif
constexpr int kSubWarps = DC_TC_SUBWARPS;  // epilogue warps per TMEM lane quarter
constexpr int kWarpBlocks = kChunkN / 64 / kSubWarps;  // 64-column blocks per epilogue warp and chunk
constexpr int kEpiWarps = 4 * kSubWarps;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kWinRow = 16;      // floats per window row: two 8-column strip slots
constexpr int kWinStride = 8 * kWinRow;      // floats per pixel
// Within a window row the four 16-byte units (slot 0 low/high, slot 1 low/high)
// are stored at unit index u ^ (pixel & 3), which spreads neighbouring pixels'
// stores and loads over the banks.
constexpr uint32_t kTmemCols = kAcc * kAccCols;
constexpr uint32_t kRowBytes = 128;  // one 128-byte K atom per operand row
static_assert(kChunkN <= kAccCols && kChunkN % 16 == 0, "MMA N");
static_assert(kChunkStrips <= 32, "one bit per strip of a chunk");
static_assert(kWarpBlocks >= 1, "every epilogue warp drains at least one 64-column block");
static_assert(kSubWarps == 2 || kSubWarps == 4, "epilogue warps per lane quarter");
static_assert(kTileM == 4 * 32, "one 4-row source gather per producer lane");

// Per-level constants of the target boxes (host-computed): a box holds br rows
// of wbox pixels (wbox a multiple of 8, br * wbox <= 256); a row wider than
// wbox is split into segs segments.
struct LevelBox {
    int wbox, br, segs;
    float inv_wbox;
};

// Per-level schedule of one tile: target rows ylo .. ylo + nrows - 1 and row
// segments sg0 .. sg0 + nsg - 1; chunks first .. first + count - 1 of the tile.
// With one segment per row a chunk holds br consecutive rows; otherwise a chunk
// is one segment of one row.
struct LevelSched {
    int first, count, ylo, nrows, sg0, nsg, pad0, pad1;
};

struct ChunkGeo {
    int y0, x0, rows, cols, n;  // first row and column, rows, real targets, MMA N
};

__device__ __forceinline__ ChunkGeo chunk_geo(const LevelSched& L, const LevelBox& B, int c) {
    ChunkGeo g;
    if (B.segs == 1) {
        g.y0 = L.ylo + c * B.br;
        g.x0 = 0;
        g.rows = min(B.br, L.ylo + L.nrows - g.y0);
    } else {
        const int r = c / L.nsg;
        g.y0 = L.ylo + r;
        g.x0 = (L.sg0 + c - r * L.nsg) * B.wbox;
        g.rows = 1;
    }
    g.cols = g.rows * B.wbox;
    g.n = (g.cols + 15) & ~15;
    return g;
}

// floor(v / d) for 0 <= v < 2^12 and 1 <= d <= 2^12 from d's reciprocal: the
// quotient of v + 0.5 is at least 0.5 / d away from an integer, far above the
// rounding error of the product.
__device__ __forceinline__ int div_small(int v, float inv_d) {
    return (int)(((float)v + 0.5f) * inv_d);
}

// The operand tensor maps: A = the 2-D store (128 source pixels x 64 channels
// boxes), B[l] = level l as [slot][H_l][W_l][C] (br x wbox x 64 boxes).
struct TcMaps {
    CUtensorMap a;
    CUtensorMap b[DC_MAX_LEVELS];
    CUtensorMap a_rows;  // the store with one-row boxes: source-tile row gathers
};

struct TcParams {
    dc::Geom g;
    LevelBox box[DC_MAX_LEVELS];
    const int* ii;
    const int* jj;
    int max_frames;
    const float* coords;
    // window-row tile order (null: source order): tile position -> source pixel,
    // per-edge flag (1: permuted), coordinates in tile-position order
    const int* perm;
    const int* pflag;
    const float* pcoords;
    float* out;
    int* err;
    int atoms;        // 128-byte K atoms per operand row (C * 2 / 128)
    uint32_t ab_fmt;  // 0 fp16, 1 bf16
    int M;            // edges
    int stall;        // test hook: withhold each CTA's first source-tile load
    long long a_off;  // source rows: 0 = the slot's (hi) rows, lo_rows = its lo copy (FP32X3)
    int accum;        // add to `out` instead of writing it (FP32X3 passes 2 and 3)
    int keep;         // a later pass reads `out` back: ordinary (L2-resident) stores
    unsigned long long wait_ns;  // limit of the pipeline waits (the drain waits keep 2 s)
};

struct TileInfo {
    int e, p0, si, sj, n, valid, gather, pad1;  // gather: source rows are permuted
};

struct Layout {
    uint32_t a, b, stage_b, win, sched, tinfo, bars, misc, strips, reps, rows, total;
};

__host__ __device__ constexpr Layout make_layout(int atoms) {
    Layout L{};
    L.a = 0;
    L.b = L.a + atoms * kTileM * kRowBytes;
    L.stage_b = atoms * kChunkN * kRowBytes;
    L.win = L.b + kStagesB * L.stage_b;
    L.sched = L.win + kTileM * kWinStride * 4;               // [2][levels] LevelSched
    L.tinfo = L.sched + 2 * DC_MAX_LEVELS * sizeof(LevelSched);
    L.bars = L.tinfo + 2 * sizeof(TileInfo);
    L.misc = L.bars + 24 * 8;
    L.strips = L.misc + 64;                                  // [levels][32] int
    L.reps = L.strips + DC_MAX_LEVELS * kChunkStrips * 4;    // [levels][33] uint
    L.rows = L.reps + DC_MAX_LEVELS * (kChunkStrips + 1) * 4;  // [128] u16: gathered pixels
    L.total = L.rows + kTileM * 2;
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
// a tile's schedule (written by the producer) is released by the MMA warp and
// every epilogue warp
constexpr int kSchedConsumers = 1 + kEpiWarps;

__device__ __forceinline__ void raise_abort(volatile int* abort, int* err, int code) {
    *abort = 1;
    atomicExch(err, code);
}

// Optional phase timers (build with -DDC_TC_PROFILE; compiled out otherwise):
// per CTA, cycles spent in each role's waits and in the epilogue phases, and a
// per-chunk event trace of CTA 0.
#ifdef DC_TC_PROFILE
__device__ unsigned long long g_tc_prof[8192 * 16];
__device__ long long g_tc_trace[8 * 1024];
#define DC_TRACE(ev, idx)                                                                  \
    do {                                                                                   \
        if (blockIdx.x == 0 && (idx) < 1024) g_tc_trace[(ev) * 1024 + (idx)] = clock64(); \
    } while (0)
#define DC_PROF_NOW() clock64()
#define DC_PROF_STORE(slot, v)                                                    \
    do {                                                                          \
        const int cta_ = blockIdx.x;                                              \
        if (cta_ < 8192) g_tc_prof[cta_ * 16 + (slot)] = (unsigned long long)(v); \
    } while (0)
#else
#define DC_TRACE(ev, idx) \
    do {                  \
    } while (0)
#define DC_PROF_NOW() 0ll
#define DC_PROF_STORE(slot, v) \
    do {                       \
    } while (0)
#endif

// All lanes of a warp wait for one barrier phase: lane 0 polls (bounded), the
// others then observe the completed phase.  Returns false on a time-out.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                          int lane, unsigned long long limit_ns) {
    int ok = 1;
    if (lane == 0) ok = mbar_wait(bar, parity, abort, limit_ns) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (ok) mbar_wait(bar, parity, abort, limit_ns);
    return ok != 0;
}

// Named barrier of the kSubWarps epilogue warps that share a TMEM lane quarter.
// Every epilogue warp waits for every accumulator phase, so a time-out ends all
// of them at the same chunk, before either meeting of that level: no warp is
// ever left alone at this barrier.
__device__ __forceinline__ void quarter_sync(int quarter) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + quarter), "r"(32 * kSubWarps) : "memory");
}

// Bilinear outputs of one pixel and level for output columns a0 .. a0 + AW - 1
// (the window columns are x offsets a, the rows y offsets b): the weights of
// batch_corr_sample_kernel (main.cu:1196-1213), evaluated separably -- first
// along x per window row (h_j = tap[a][j] wx0 + tap[a+1][j] wx1), then along y
// (h_b (1 - dy) + h_{b+1} dy) -- which takes 30 instead of 50 operations per
// output column; the rounding differs from the reference's four-term chain by
// a few fp32 ulps, far inside the fused path's tolerance (its dot products
// are tensor-core sums anyway).  The window holds raw dot products, so alpha
// rides on the x weights.  kCheck: some taps may lie outside the level; they
// read as +0, as skipping them does in the reference; so do all taps of a
// pixel with no window in the level (any false).
template <int R, int AW, bool kCheck>
__device__ __forceinline__ void bilinear_columns(const float* win, int swz, int kx, int a0, int bx,
                                                 int by, int Wl, int Hl, bool any, float dx,
                                                 float dy, float alpha, float* ol, int hw,
                                                 bool accum, bool keep,
                                                 const float (&old)[AW][2 * R + 1]) {
    constexpr int D = 2 * R + 1, NW = 2 * R + 2;
    bool vy[NW];
#pragma unroll
    for (int k = 0; k < NW; k++) vy[k] = !kCheck || (any && (unsigned)(by + k) < (unsigned)Hl);
    const float ux = alpha * (1.0f - dx), vx_w = alpha * dx;
    const float uy = 1.0f - dy;
    float pu[NW];
#pragma unroll
    for (int ii = 0; ii <= AW; ii++) {
        const int ix = min(a0 + ii, NW - 1);
        const bool vx = a0 + ii < NW && (!kCheck || (unsigned)(bx + ix) < (unsigned)Wl);
        // window column ix = row column kx + ix (0..14), swizzled unit
        const int col = kx + ix;
        const float* wc = win + (((col >> 2) ^ swz) << 2) + (col & 3);
        float tap[NW];
#pragma unroll
        for (int j = 0; j < NW; j++) {
            if (kCheck)
                tap[j] = (vx && vy[j]) ? wc[j * kWinRow] : 0.0f;
            else
                tap[j] = wc[j * kWinRow];
        }
        if (ii > 0 && a0 + ii - 1 < D) {
            float* o = ol + (size_t)((a0 + ii - 1) * D) * hw;
            // separable: interpolate along x per window row, then along y
            float hx[NW];
#pragma unroll
            for (int j = 0; j < NW; j++) hx[j] = fmaf(tap[j], vx_w, pu[j]);
#pragma unroll
            for (int b = 0; b < D; b++) {
                float acc = fmaf(hx[b + 1], dy, hx[b] * uy);
                if (accum) acc = old[ii - 1][b] + acc;  // FP32X3 passes 2, 3 add their products
                if (keep)
                    *o = acc;  // read again by the next FP32X3 pass: keep it in L2
                else
                    __stcs(o, acc);
                o += hw;
            }
        }
#pragma unroll
        for (int j = 0; j < NW; j++) pu[j] = tap[j] * ux;
    }
}

// The outputs an FP32X3 pass adds to (columns a0 .. a0 + AW - 1), loaded before
// the level's window barrier so that their latency hides behind it.
template <int R, int AW>
__device__ __forceinline__ void load_old(const float* ol, int a0, int hw,
                                         float (&old)[AW][2 * R + 1]) {
    constexpr int D = 2 * R + 1;
#pragma unroll
    for (int ii = 0; ii < AW; ii++)
#pragma unroll
        for (int b = 0; b < D; b++)
            old[ii][b] = a0 + ii < D ? __ldcs(ol + (size_t)((a0 + ii) * D + b) * hw) : 0.0f;
}

// Persistent: CTA b handles tiles b, b + gridDim.x, ...; tile t = (edge t / tpe,
// source pixels 128 * (t % tpe) ..).
// kSplit: a pass of DC_PREC_FP32X3 (may add to `out` and keep it in L2); the
// other precisions run the variant without that code.
template <int R, bool kSplit>
__global__ void __launch_bounds__(kThreads, 1)
    corr_tc_kernel(const __grid_constant__ TcMaps maps, TcParams P) {
    constexpr int D = 2 * R + 1, NW = 2 * R + 2;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base by pointer arithmetic on the shared array itself, so
    // that the compiler keeps the shared address space (LDS/STS, not generic)
    uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
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
            mbar_init(bar(kBarSEmpty + b), kSchedConsumers);
        }
        misc[kMiscAbort] = 0;
        fence_mbar_init();
        tma_prefetch_desc(&maps.a);
        for (int l = 0; l < g.levels; l++) tma_prefetch_desc(&maps.b[l]);
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(misc + kMiscTmem), kTmemCols);
        tmem_relinquish();
    }
    // Per-level tables of the chunk strips (strip q = TMEM columns 8q .. 8q + 7):
    // strip_tab[l][q] = its row within the chunk (low half) and its strip within
    // the row segment (high half); rep_tab[l][r] = the bit mask of strips 0 of
    // rows 0 .. r - 1 (rows are spr = wbox / 8 strips apart).
    int* strip_tab = reinterpret_cast<int*>(base + Ly.strips);
    unsigned* rep_tab = reinterpret_cast<unsigned*>(base + Ly.reps);
    if (threadIdx.x < DC_MAX_LEVELS * kChunkStrips) {
        const int l = threadIdx.x / kChunkStrips, n = kStrip * (threadIdx.x % kChunkStrips);
        const LevelBox& B = P.box[l];
        const int r = div_small(n, B.inv_wbox);
        strip_tab[threadIdx.x] = r | (((n - r * B.wbox) >> 3) << 16);
    } else if (threadIdx.x < DC_MAX_LEVELS * kChunkStrips + DC_MAX_LEVELS * (kChunkStrips + 1)) {
        const int idx = threadIdx.x - DC_MAX_LEVELS * kChunkStrips;
        const int l = idx / (kChunkStrips + 1), r = idx % (kChunkStrips + 1);
        const int spr = P.box[l].wbox / kStrip;
        unsigned m = 0;
        for (int i = 0; i < r && i * spr < kChunkStrips; i++) m |= 1u << (i * spr);
        rep_tab[idx] = m;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = (uint32_t)misc[kMiscTmem];
    long long w_a = 0, w_b = 0, w_c = 0;  // phase cycles (profiling builds)

    if (warp == 0) {
        // ---- producer: per tile, the schedule (target rows, and row segments, of
        //      each level that some window of the tile's pixels touches, from
        //      coordinates loaded one tile ahead), then the source tile and the
        //      target-row chunks through TMA (one elected lane)
        int gc = 0, na = 0, i = 0;
        int a_issued = 0, a_parity = 0, last_gc = 0;
        float cxn[kTileM / 32], cyn[kTileM / 32];
        int pxn[kTileM / 32];
        int sin_ = -1, sjn = -1, gan = 0;
        const float* const cbase = P.perm ? P.pcoords : P.coords;
        unsigned short* const arows = reinterpret_cast<unsigned short*>(base + Ly.rows);
#define DC_TC_LOAD_COORDS(tt)                                                      \
    do {                                                                           \
        _Pragma("unroll") for (int k = 0; k < kTileM / 32; k++) {                  \
            cxn[k] = cyn[k] = 0.0f;                                                \
            pxn[k] = 0;                                                            \
        }                                                                          \
        if ((tt) < ntiles) {                                                       \
            const int e_ = (tt) / tpe, q0_ = ((tt) - e_ * tpe) * kTileM;           \
            sin_ = __ldg(P.ii + e_);                                               \
            sjn = __ldg(P.jj + e_);                                                \
            gan = P.perm ? __ldg(P.pflag + e_) : 0;                                \
            _Pragma("unroll") for (int k = 0; k < kTileM / 32; k++) {              \
                const int q_ = q0_ + lane + 32 * k;                                \
                if (q_ < hw) {                                                     \
                    cxn[k] = __ldg(cbase + (size_t)e_ * 2 * hw + q_);              \
                    cyn[k] = __ldg(cbase + (size_t)e_ * 2 * hw + hw + q_);         \
                    if (P.perm) pxn[k] = __ldg(P.perm + (size_t)e_ * hw + q_);     \
                }                                                                  \
            }                                                                      \
        }                                                                          \
    } while (0)
        DC_TC_LOAD_COORDS(blockIdx.x);  // all loads of a tile in flight at once
        for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x, i++) {
            const int tb = i & 1;
            if (i >= 2 && !warp_wait(bar(kBarSEmpty + tb), ((i >> 1) - 1) & 1, abort, lane, P.wait_ns)) {
                if (lane == 0) raise_abort(abort, P.err, 1);
                break;
            }
            float cx[kTileM / 32], cy[kTileM / 32];
            const int ga = gan;
#pragma unroll
            for (int k = 0; k < kTileM / 32; k++) {
                cx[k] = cxn[k];
                cy[k] = cyn[k];
                // the source rows to gather (lane L reads rows 4L .. 4L + 3 below)
                if (ga) arows[lane + 32 * k] = (unsigned short)pxn[k];  // hw <= DC_MAX_HW < 2^16
            }
            const int si = sin_, sj = sjn;
            DC_TC_LOAD_COORDS(t + gridDim.x);
            const int e = t / tpe, p0 = (t - e * tpe) * kTileM;
            const bool valid = si >= 0 && si < P.max_frames && sj >= 0 && sj < P.max_frames;
            int n = 0;
            // one level at a time (a rolled loop: the producer shares its SM
            // sub-partition's instruction cache with two epilogue warps)
#pragma unroll 1
            for (int l = 0; l < DC_MAX_LEVELS; l++) {
                int ylo_ = 0x7fffffff, yhi_ = -1, xlo_ = 0x7fffffff, xhi_ = -1;
                if (l < g.levels) {
                    const float sc = 1.0f / (float)(1 << l);
#pragma unroll
                    for (int k = 0; k < kTileM / 32; k++) {
                        if (!(valid && p0 + lane + 32 * k < hw)) continue;
                        const int by = (int)floorf(cy[k] * sc) - R, bx = (int)floorf(cx[k] * sc) - R;
                        const int a0 = max(by, 0), a1 = min(by + NW - 1, g.H[l] - 1);
                        const int b0 = max(bx, 0), b1 = min(bx + NW - 1, g.W[l] - 1);
                        if (a0 <= a1 && b0 <= b1) {
                            ylo_ = min(ylo_, a0);
                            yhi_ = max(yhi_, a1);
                            xlo_ = min(xlo_, b0);
                            xhi_ = max(xhi_, b1);
                        }
                    }
                }
                const int ylo = __reduce_min_sync(0xffffffffu, ylo_);
                const int yhi = __reduce_max_sync(0xffffffffu, yhi_);
                const int xlo = __reduce_min_sync(0xffffffffu, xlo_);
                const int xhi = __reduce_max_sync(0xffffffffu, xhi_);
                LevelSched L;
                L.first = n;
                L.count = 0;
                L.ylo = ylo;
                L.nrows = 0;
                L.sg0 = 0;
                L.nsg = 1;
                L.pad0 = L.pad1 = 0;
                if (l < g.levels && ylo <= yhi) {
                    const LevelBox& B = P.box[l];
                    L.nrows = yhi - ylo + 1;
                    if (B.segs == 1) {
                        L.count = (L.nrows + B.br - 1) / B.br;
                    } else {
                        L.sg0 = xlo / B.wbox;
                        L.nsg = xhi / B.wbox - L.sg0 + 1;
                        L.count = L.nrows * L.nsg;
                    }
                }
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
                ti.gather = ga;
                ti.pad1 = 0;
                tinfo[tb] = ti;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarSFull + tb));  // release: schedule
            const TileInfo ti = tinfo[tb];
            const LevelSched* sch = sched_base + tb * DC_MAX_LEVELS;
            if (ti.n > 0) {
                // The first kStagesB target-row chunks do not depend on the single
                // source-tile buffer: issue them first, so their loads overlap the
                // previous tile's last MMAs; then wait until those MMAs release the
                // source buffer and load this tile's source pixels; then the rest.
                const int pre = min(kStagesB, ti.n);
                int lv = 0, ok = 1;
                // (lane 0) target-row chunk c of this tile into the next stage
                auto issue_chunk = [&](int c) -> int {
                    while (c >= sch[lv].first + sch[lv].count) lv++;
                    const int s = gc % kStagesB;
                    const long long t0 = DC_PROF_NOW();
                    if (gc >= kStagesB &&
                        !mbar_wait(bar(kBarEmpty + s), ((gc / kStagesB) - 1) & 1, abort, P.wait_ns)) {
                        raise_abort(abort, P.err, 4);
                        return 0;
                    }
                    w_a += DC_PROF_NOW() - t0;
                    DC_TRACE(0, gc);
                    const LevelBox& B = P.box[lv];
                    const ChunkGeo cg = chunk_geo(sch[lv], B, c - sch[lv].first);
                    mbar_arrive_expect_tx(bar(kBarFull + s), P.atoms * B.wbox * B.br * kRowBytes);
                    for (int k = 0; k < P.atoms; k++)
                        tma_load_4d(sB + s * Ly.stage_b + k * kChunkN * kRowBytes, &maps.b[lv],
                                    k * 64, cg.x0, cg.y0, ti.sj, bar(kBarFull + s));
                    gc++;
                    last_gc = gc;
                    return 1;
                };
                if (lane == 0)
                    for (int c = 0; c < pre && ok; c++) ok = issue_chunk(c);
                int aload = 0;
                if (lane == 0 && ok) {
                    if (na >= 1 && !mbar_wait(bar(kBarAEmpty), (na - 1) & 1, abort, P.wait_ns)) {
                        raise_abort(abort, P.err, 3);
                        ok = 0;
                    } else if (!(P.stall && na == 0)) {
                        mbar_arrive_expect_tx(bar(kBarAFull), P.atoms * kTileM * kRowBytes);
                        a_issued = 1;
                        a_parity = na & 1;
                        aload = 1;
                    }
                }
                // (the shuffles also order lane 0's expect-tx before the gathers)
                ok = __shfl_sync(0xffffffffu, ok, 0);
                aload = __shfl_sync(0xffffffffu, aload, 0);
                if (aload) {
                    const int rbase = (int)((long long)ti.si * g.frame_rows + P.a_off + g.row0[0]);
                    if (ti.gather) {
                        // permuted tile: lane L gathers source rows 4L .. 4L + 3 (512
                        // bytes per K atom), all lanes at once
                        const int r0 = rbase + arows[4 * lane], r1 = rbase + arows[4 * lane + 1];
                        const int r2 = rbase + arows[4 * lane + 2], r3 = rbase + arows[4 * lane + 3];
                        for (int k = 0; k < P.atoms; k++)
                            tma_gather4(sA + k * kTileM * kRowBytes + lane * 4 * kRowBytes,
                                        &maps.a_rows, k * 64, r0, r1, r2, r3, bar(kBarAFull));
                    } else if (lane == 0) {
                        for (int k = 0; k < P.atoms; k++)
                            tma_load_2d(sA + k * kTileM * kRowBytes, &maps.a, k * 64,
                                        rbase + ti.p0, bar(kBarAFull));
                    }
                }
                if (lane == 0 && ok)
                    for (int c = pre; c < ti.n && ok; c++) ok = issue_chunk(c);
            }
            if (ti.n > 0) na++;
            __syncwarp();
        }
        (void)arows;
        if (lane == 0) {
            DC_PROF_STORE(4, w_a);
            if (*abort) {
                // let this CTA's copies in flight land before the CTA exits
                if (a_issued) mbar_wait(bar(kBarAFull), a_parity, nullptr);
                for (int c = max(0, last_gc - kStagesB); c < last_gc; c++)
                    mbar_wait(bar(kBarFull + c % kStagesB), (c / kStagesB) & 1, nullptr);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer
        int gc = 0, na = 0, i = 0;
        int last_mma = -1;  // global chunk index of the last committed MMA group
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, i++) {
            const int tb = i & 1;
            if (!warp_wait(bar(kBarSFull + tb), (i >> 1) & 1, abort, lane, P.wait_ns)) {
                if (lane == 0) raise_abort(abort, P.err, 5);
                break;
            }
            const TileInfo ti = tinfo[tb];
            const LevelSched* sch = sched_base + tb * DC_MAX_LEVELS;
            bool ok = true;
            if (lane == 0 && ti.n > 0) {
                if (!mbar_wait(bar(kBarAFull), na & 1, abort, P.wait_ns)) {
                    raise_abort(abort, P.err, 6);
                    ok = false;
                } else {
                    tc_fence_after();
                    const int ksteps = P.atoms * 4;  // 16 elements (32 bytes) per MMA
                    int lv = 0;
                    for (int c = 0; c < ti.n; c++, gc++) {
                        while (c >= sch[lv].first + sch[lv].count) lv++;
                        const int s = gc % kStagesB, a = gc % kAcc;
                        const long long t0 = DC_PROF_NOW();
                        if (!mbar_wait(bar(kBarFull + s), (gc / kStagesB) & 1, abort, P.wait_ns)) {
                            raise_abort(abort, P.err, 7);
                            ok = false;
                            break;
                        }
                        const long long t1 = DC_PROF_NOW();
                        w_a += t1 - t0;
                        DC_TRACE(1, gc);
                        if (gc >= kAcc &&
                            !mbar_wait(bar(kBarTEmpty + a), ((gc / kAcc) - 1) & 1, abort, P.wait_ns)) {
                            raise_abort(abort, P.err, 8);
                            ok = false;
                            break;
                        }
                        w_b += DC_PROF_NOW() - t1;
                        DC_TRACE(2, gc);
                        tc_fence_after();
                        const int nn = chunk_geo(sch[lv], P.box[lv], c - sch[lv].first).n;
                        const uint32_t idesc = idesc_f16(P.ab_fmt, kTileM, nn);
                        const uint32_t d = tmem + (uint32_t)(a * kAccCols);
                        for (int kk = 0; kk < ksteps; kk++) {
                            const int at = kk >> 2, wi = kk & 3;
                            const uint64_t ad = sdesc_sw128(sA + at * kTileM * kRowBytes + wi * 32);
                            const uint64_t bd = sdesc_sw128(sB + s * Ly.stage_b +
                                                            at * kChunkN * kRowBytes + wi * 32);
                            mma_f16(d, ad, bd, idesc, kk > 0 ? 1u : 0u);
                        }
                        mma_commit(bar(kBarEmpty + s));
                        mma_commit(bar(kBarTFull + a));
                        last_mma = gc;
                        DC_TRACE(3, gc);
                    }
                    mma_commit(bar(kBarAEmpty));  // the source tile may be replaced
                }
            }
            if (ti.n > 0) na++;
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (lane == 0) mbar_arrive(bar(kBarSEmpty + tb));
            if (!ok) break;
        }
        if (lane == 0 && *abort && last_mma >= 0) {
            // the MMAs issued so far read shared memory and write TMEM: let them
            // finish (bounded) before the CTA frees TMEM and exits
            mbar_wait(bar(kBarEmpty + last_mma % kStagesB), (last_mma / kStagesB) & 1, nullptr);
        }
        if (lane == 0) {
            DC_PROF_STORE(2, w_a);
            DC_PROF_STORE(3, w_b);
            DC_PROF_STORE(8, gc);
            DC_PROF_STORE(9, i);
        }
        __syncwarp();
    } else {
        // ---- epilogue: the kSubWarps warps of a TMEM lane quarter take
        //      256 / kSubWarps columns of every chunk each and split the outputs
        const int quarter = warp & 3;       // TMEM lane quarter of this warp
        const int sub = (warp - 2) >> 2;    // which loads / output columns (0..kSubWarps-1)
        const int ti_px = 32 * quarter + lane;
        float* win = win_base + ti_px * kWinStride;
        const uint32_t win_s = smem_addr(win);
        const int swz = ti_px & 3;  // unit swizzle of this pixel's window rows
        const uint32_t tl = tmem + ((uint32_t)(32 * quarter) << 16);
        int gc = 0, i = 0;
        bool alive = true;
        // this pixel's coordinates, loaded one tile ahead
        // (window-row order: the coordinates in tile-position order; outputs are
        // written at the tile position and moved to their pixel by
        // unpermute_rows_kernel after the call's passes)
        float cx_next = 0.0f, cy_next = 0.0f;
        const float* const cbase = P.perm ? P.pcoords : P.coords;
#define DC_TC_PIXEL_COORDS(tt)                                               \
    do {                                                                     \
        cx_next = cy_next = 0.0f;                                            \
        if ((tt) < ntiles) {                                                 \
            const int e_ = (tt) / tpe, q_ = ((tt) - e_ * tpe) * kTileM + ti_px; \
            if (q_ < hw) {                                                   \
                cx_next = __ldg(cbase + (size_t)e_ * 2 * hw + q_);           \
                cy_next = __ldg(cbase + (size_t)e_ * 2 * hw + hw + q_);      \
            }                                                                \
        }                                                                    \
    } while (0)
        DC_TC_PIXEL_COORDS(blockIdx.x);
        for (int t = blockIdx.x; t < ntiles && alive; t += gridDim.x, i++) {
            const int tb = i & 1;
            const float cx = cx_next, cy = cy_next;
            DC_TC_PIXEL_COORDS(t + gridDim.x);
            const long long t0s = DC_PROF_NOW();
            if (!warp_wait(bar(kBarSFull + tb), (i >> 1) & 1, abort, lane, P.wait_ns)) {
                if (lane == 0) raise_abort(abort, P.err, 9);
                break;
            }
            w_a += DC_PROF_NOW() - t0s;
            const TileInfo tinf = tinfo[tb];
            const LevelSched* sch = sched_base + tb * DC_MAX_LEVELS;
            const int p = tinf.p0 + ti_px;  // tile position = pixel in source order
            const bool pv = p < hw;
            const bool valid = tinf.valid != 0;
            float* out_e = P.out + (size_t)tinf.e * nch * hw;
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
                const LevelBox B = P.box[l];
                // the window's first column lies in strip s0 (at column kx of it);
                // strips s0 and s0 + 1 go to window slots 0 and 1
                const int s0 = bx >> 3, kx = bx & 7;
                const int* strip_l = strip_tab + l * kChunkStrips;
                const unsigned* rep_l = rep_tab + l * (kChunkStrips + 1);
                const int spr = B.wbox / kStrip;
                for (int c = 0; c < Ls.count; c++, gc++) {
                    const int a = gc % kAcc;
                    const long long t0 = DC_PROF_NOW();
                    if (!warp_wait(bar(kBarTFull + a), (gc / kAcc) & 1, abort, lane, P.wait_ns)) {
                        if (lane == 0) raise_abort(abort, P.err, 10);
                        alive = false;
                        break;
                    }
                    tc_fence_after();
                    const long long t1 = DC_PROF_NOW();
                    w_a += t1 - t0;
                    if (lane == 0 && warp == 2) DC_TRACE(4, gc);
                    const ChunkGeo cg = chunk_geo(Ls, B, c);
                    // bit q of m: strip q of this chunk holds part of this pixel's
                    // window -- rows ra .. rb of the chunk, strips xs0 and xs0 + 1
                    // of the row segment
                    unsigned m = 0;
                    const int ry = cg.y0 - by, xs0 = s0 - (cg.x0 >> 3);
                    const int ra = max(-ry, 0), rb = min(NW - 1 - ry, cg.rows - 1);
                    if (any && ra <= rb) {
                        const unsigned rr = rep_l[rb + 1] ^ rep_l[ra];
                        if ((unsigned)xs0 < (unsigned)spr) m |= rr << xs0;
                        if ((unsigned)(xs0 + 1) < (unsigned)spr) m |= rr << (xs0 + 1);
                    }
                    // this warp's 64-column blocks: chunk strips 8 * (kWarpBlocks * sub + bb) ..
                    // (not unrolled: the smaller instruction footprint is 3 % faster)
#pragma unroll 1
                    for (int bb = 0; bb < kWarpBlocks; bb++) {
                        const int blk = kWarpBlocks * sub + bb;
                        if (64 * blk >= cg.cols) break;
                        const unsigned n8 = (m >> (8 * blk)) & 0xffu;
                        if (!__any_sync(0xffffffffu, n8 != 0)) continue;
                        float v[64];
                        tmem_ld64(tl + (uint32_t)(a * kAccCols + 64 * blk), v);
                        if (lane == 0 && warp == 2) DC_TRACE(5 + bb, gc);
#pragma unroll
                        for (int k = 0; k < 8; k++) {
                            // predicated stores: no per-strip branch
                            const bool need = (n8 >> k) & 1u;
                            const int e = strip_l[8 * blk + k];
                            const int wr = ry + (e & 0xffff);
                            const int u = 2 * ((e >> 16) - xs0);
                            const uint32_t row = win_s + (uint32_t)(wr * kWinRow) * 4u;
                            st_shared_v4_if(need, row + (uint32_t)((u ^ swz) << 4), v[8 * k + 0],
                                            v[8 * k + 1], v[8 * k + 2], v[8 * k + 3]);
                            st_shared_v4_if(need, row + (uint32_t)(((u + 1) ^ swz) << 4),
                                            v[8 * k + 4], v[8 * k + 5], v[8 * k + 6],
                                            v[8 * k + 7]);
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(bar(kBarTEmpty + a));
                    if (lane == 0 && warp == 2) DC_TRACE(7, gc);
                    w_b += DC_PROF_NOW() - t1;
                }
                if (!alive) break;
                const long long t2 = DC_PROF_NOW();
                constexpr int AW = (D + kSubWarps - 1) / kSubWarps;  // 4, 3 at R = 3
                float* ol = out_e + (size_t)(l * D * D) * hw + p;
                float old[AW][D];
                const bool accum = kSplit && P.accum, keep = kSplit && P.keep;
                if (accum && pv) load_old<R, AW>(ol, sub * AW, hw, old);
                quarter_sync(quarter);  // all strips of this level are in the windows
                // one (checked) variant only: a second, unchecked copy for
                // interior windows made the kernel 3 % slower -- the epilogue is
                // sensitive to its instruction footprint
                if (pv)
                    bilinear_columns<R, AW, true>(win, swz, kx, sub * AW, bx, by, Wl, Hl, any, dx,
                                                  dy, g.alpha, ol, hw, accum, keep, old);
                quarter_sync(quarter);  // all are done reading before the next level
                w_c += DC_PROF_NOW() - t2;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(kBarSEmpty + tb));
        }
        if (lane == 0 && warp == 2) {
            DC_PROF_STORE(5, w_a);
            DC_PROF_STORE(6, w_b);
            DC_PROF_STORE(7, w_c);
        }
    }

#undef DC_TC_LOAD_COORDS
#undef DC_TC_PIXEL_COORDS
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (threadIdx.x == 0) DC_PROF_STORE(0, DC_PROF_NOW() - t_start);
}

// ---- window-row tile order (dc_set_tile_order) -------------------------------
// One CTA per edge sorts the edge's source pixels by the row of their level-0
// window, key = floor(y) clamped to [-kBinPad, H0 + kBinPad - 1]: a counting
// sort, stable (ties in pixel order), deterministic.  Warp w owns a contiguous
// segment of pixels; cnt[key][w] counts, an exclusive scan in (key, warp) order
// turns the counts into each warp's first position per key, and each warp then
// places its pixels in order (__match_any_sync ranks equal keys within 32).
// The kernel also estimates, for both orders, the target rows the fused kernel
// would stream (per 128-pixel tile: key span + 2r + 2) and, for DC_ORDER_AUTO,
// keeps the window-row order only where it saves enough (kAutoPxPerChannel).  It
// writes the permutation, the flag, and the coordinates in position order.
constexpr int kBinThreads = 1024;
constexpr int kBinPad = 8;
constexpr int kBinMaxKeys = 512;
// DC_ORDER_AUTO keeps the window-row order where the level-0 target pixels it
// saves per 128-pixel tile (estimated rows saved x W0) reach kAutoPxPerChannel
// x the output channels: the gain grows with the target pixels no longer
// multiplied, the cost (reordering the tile's outputs, one read and one write
// of 128 x channels floats) with the channels.  Measured on one B200 (fp16,
// 196 channels, so a threshold of 1568), window-row against source order:
// ~530 pixels saved per tile (48x64, flow noise N(0, 2 px)): 1.4x slower;
// ~1350 (54x96, N(0, 3 px)): 1.03x faster; ~2200 (48x64, N(0, 8 px)): 1.12x
// faster; ~3500 (54x96, N(0, 8 px)): 1.6x faster.
constexpr int kAutoPxPerChannel = 8;

__device__ __forceinline__ int bin_key(float y, int H0) {
    // fmaxf / fminf return the other operand for a NaN: NaN sorts first
    const float yc = fminf(fmaxf(y, -(float)kBinPad), (float)(H0 + kBinPad - 1));
    return (int)floorf(yc) + kBinPad;
}

__global__ void __launch_bounds__(kBinThreads)
    tile_order_kernel(const float* coords, int hw, int H0, int W0, int nch, int R, int order,
                      int* perm, int* pflag, float* pcoords) {
    extern __shared__ int cnt[];  // [nkeys][32]
    __shared__ int warp_tot[32];
    __shared__ int cost[2];       // target rows summed over tiles: source, window-row order
    const int e = blockIdx.x, nkeys = H0 + 2 * kBinPad;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* cx = coords + (size_t)e * 2 * hw;
    const float* cy = cx + hw;
    int* pe = perm + (size_t)e * hw;
    float* qx = pcoords + (size_t)e * 2 * hw;
    float* qy = qx + hw;
    const int seg = ((hw + 31) / 32 + 31) & ~31;  // pixels per warp, a multiple of 32
    const int beg = min(warp * seg, hw), end = min(beg + seg, hw);
    const int ntile = (hw + 127) / 128;
    for (int i = threadIdx.x; i < nkeys * 32; i += kBinThreads) cnt[i] = 0;
    if (threadIdx.x < 2) cost[threadIdx.x] = 0;
    __syncthreads();
    for (int p = beg + lane; p < end; p += 32) atomicAdd(&cnt[bin_key(cy[p], H0) * 32 + warp], 1);
    for (int t = warp; t < ntile; t += 32) {
        int lo = 0x7fffffff, hi = -1;
        for (int k = 0; k < 4; k++) {
            const int p = 128 * t + lane + 32 * k;
            if (p < hw) {
                const int key = bin_key(cy[p], H0);
                lo = min(lo, key);
                hi = max(hi, key);
            }
        }
        lo = __reduce_min_sync(0xffffffffu, lo);
        hi = __reduce_max_sync(0xffffffffu, hi);
        if (lane == 0) atomicAdd(&cost[0], hi - lo + 2 * R + 2);
    }
    __syncthreads();
    // exclusive scan of cnt in (key, warp) order: per thread a run of entries
    const int n = nkeys * 32, per = (n + kBinThreads - 1) / kBinThreads;
    const int i0 = min(threadIdx.x * per, n), i1 = min(i0 + per, n);
    int run_sum = 0;
    for (int i = i0; i < i1; i++) run_sum += cnt[i];
    int inc = run_sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, d);
        if (lane >= d) inc += v;
    }
    if (lane == 31) warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const int v = warp_tot[lane];
        int wi = v;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, wi, d);
            if (lane >= d) wi += u;
        }
        warp_tot[lane] = wi - v;
    }
    __syncthreads();
    int run = warp_tot[warp] + inc - run_sum;
    for (int i = i0; i < i1; i++) {
        const int c = cnt[i];
        cnt[i] = run;
        run += c;
    }
    __syncthreads();
    // key of sorted position s: the last key whose first position is <= s
    auto key_at = [&](int s_) {
        int lo = 0, hi = nkeys - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (cnt[mid * 32] <= s_) lo = mid; else hi = mid - 1;
        }
        return lo;
    };
    for (int t = threadIdx.x; t < ntile; t += kBinThreads) {
        const int s0 = 128 * t, s1 = min(s0 + 128, hw) - 1;
        atomicAdd(&cost[1], key_at(s1) - key_at(s0) + 2 * R + 2);
    }
    __syncthreads();
    const bool binned = order == DC_ORDER_WINDOW_ROW ||
                        (order == DC_ORDER_AUTO &&
                         (long long)(cost[0] - cost[1]) * W0 >=
                             (long long)kAutoPxPerChannel * nch * ntile);
    if (threadIdx.x == 0) pflag[e] = binned ? 1 : 0;
    if (!binned) {
        for (int p = threadIdx.x; p < hw; p += kBinThreads) {
            pe[p] = p;
            qx[p] = cx[p];
            qy[p] = cy[p];
        }
        return;
    }
    for (int p0 = beg; p0 < end; p0 += 32) {
        const int p = p0 + lane;
        const bool act = p < end;
        const unsigned am = __ballot_sync(0xffffffffu, act);
        if (act) {
            const float y = cy[p];
            const int key = bin_key(y, H0);
            const unsigned peers = __match_any_sync(am, key);
            const int rank = __popc(peers & ((1u << lane) - 1u));
            int* slot = &cnt[key * 32 + warp];
            const int pos = *slot + rank;
            pe[pos] = p;
            qx[pos] = cx[p];
            qy[pos] = y;
            __syncwarp(am);
            if (rank == 0) *slot += __popc(peers);
        }
        __syncwarp();
    }
}

// Window-row order, after the fused kernel: row (e, ch) of `out` holds its
// values in tile-position order; move them to pixel order in place (one CTA
// per row: the row through shared memory, so that both global passes are
// coalesced).  A CTA takes kUnpermRows rows of one edge (grid: edges x row
// groups), so the CTAs of edges left in source order (flag 0), which return at
// once, are few.
constexpr int kUnpermThreads = 256;
constexpr int kUnpermRows = 7;
__global__ void __launch_bounds__(kUnpermThreads)
    unpermute_rows_kernel(float* out, int nch, int hw, const int* perm, const int* pflag) {
    extern __shared__ float row_s[];  // [hw], pixel order
    const int e = blockIdx.x;
    if (!__ldg(pflag + e)) return;
    const int* pe = perm + (size_t)e * hw;
    const int ch1 = min(nch, (int)(blockIdx.y + 1) * kUnpermRows);
    for (int ch = blockIdx.y * kUnpermRows; ch < ch1; ch++) {
        float* row = out + ((size_t)e * nch + ch) * hw;
        __syncthreads();  // the previous row's stores have read row_s
        if ((hw & 3) == 0) {
            // rows start 16-byte aligned: 4 values (and 4 pixel indices) per access
            const int n4 = hw >> 2;
            const float4* row4 = reinterpret_cast<const float4*>(row);
            const int4* pe4 = reinterpret_cast<const int4*>(pe);
            for (int i = threadIdx.x; i < n4; i += kUnpermThreads) {
                const float4 v = __ldcs(row4 + i);
                const int4 q = __ldg(pe4 + i);
                row_s[q.x] = v.x;
                row_s[q.y] = v.y;
                row_s[q.z] = v.z;
                row_s[q.w] = v.w;
            }
            __syncthreads();
            float4* out4 = reinterpret_cast<float4*>(row);
            for (int i = threadIdx.x; i < n4; i += kUnpermThreads)
                __stcs(out4 + i, reinterpret_cast<const float4*>(row_s)[i]);
        } else {
            for (int s_ = threadIdx.x; s_ < hw; s_ += kUnpermThreads)
                row_s[__ldg(pe + s_)] = __ldcs(row + s_);
            __syncthreads();
            for (int p = threadIdx.x; p < hw; p += kUnpermThreads) __stcs(row + p, row_s[p]);
        }
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

// Target boxes of level l: rows padded to a multiple of 8 pixels; a box holds
// as many whole rows as fit in kChunkN targets, or one kChunkN-wide segment of
// a wider row.
LevelBox level_box(const dc_ctx* ctx, int l) {
    LevelBox b;
    const int wpad = (ctx->W[l] + kStrip - 1) / kStrip * kStrip;
    b.wbox = wpad < kChunkN ? wpad : kChunkN;
    b.br = kChunkN / b.wbox;
    b.segs = (wpad + b.wbox - 1) / b.wbox;
    b.inv_wbox = 1.0f / (float)b.wbox;
    return b;
}

// Process-wide test hook of the bounded waits (dc_debug_inject_stall)
// (> 0: stall active, with this wait limit in ns)
std::atomic<long long> g_test_wait_ns{0};

}  // namespace

extern "C" int dc_debug_inject_stall(long long wait_limit_ns) {
    if (wait_limit_ns < 0) return DC_ERR_INVALID_ARG;
    g_test_wait_ns.store(wait_limit_ns);
    return DC_OK;
}

#ifdef DC_TC_PROFILE
extern "C" int dc_tc_profile_read(unsigned long long* host, int n) {
    return (int)cudaMemcpyFromSymbol(host, g_tc_prof, sizeof(unsigned long long) * n);
}
extern "C" int dc_tc_trace_read(long long* host) {
    return (int)cudaMemcpyFromSymbol(host, g_tc_trace, sizeof(long long) * 8 * 1024);
}
#endif

int dc_tmap_2d_f32(void* tmap, const void* base, unsigned long long cols,
                   unsigned long long rows, unsigned box_cols, unsigned box_rows) {
    EncodeTiledFn enc = get_encode();
    if (!enc) return DC_ERR_CUDA;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(reinterpret_cast<CUtensorMap*>(tmap), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                           const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? DC_OK : DC_ERR_CUDA;
}

bool dc_tc_supported(const dc_ctx* ctx) {
    const int p = ctx->cfg.precision;
    return (p == DC_PREC_FP16 || p == DC_PREC_BF16 || p == DC_PREC_TF32 || p == DC_PREC_FP32X3) &&
           (ctx->cfg.channels == 64 || ctx->cfg.channels == 128);
}

// Tensor maps over the store of 16-bit elements, all with 128-byte swizzle (the
// canonical K-major operand layout of tcgen05): A = [max_frames * frame_rows][C]
// with boxes of 128 rows x 64 channels; B[l] = level l as the 4-D tensor
// [slot][H_l][W_l][C] (a slot's level-l rows start at level_row0[l], slots are
// frame_rows apart) with boxes of br rows x wbox pixels x 64 channels, pixels
// outside the level reading as zeros (out-of-bounds fill).
int dc_tc_prepare(dc_ctx* ctx) {
    EncodeTiledFn enc = get_encode();
    if (!enc) return dc_fail(ctx, DC_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const CUtensorMapDataType dt = ctx->cfg.precision == DC_PREC_BF16
                                       ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const size_t row_bytes = (size_t)ctx->cfg.channels * 2;
    cuuint64_t dims[2] = {(cuuint64_t)ctx->cfg.channels,
                          (cuuint64_t)ctx->cfg.max_frames * ctx->frame_rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t estr[2] = {1, 1};
    cuuint32_t box[2] = {64, (cuuint32_t)kTileM};
    CUresult r1 = enc(reinterpret_cast<CUtensorMap*>(ctx->tmap_a), dt, 2, ctx->store, dims,
                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r1 != CUDA_SUCCESS) return dc_fail(ctx, DC_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    cuuint32_t box_row[2] = {64, 1};
    CUresult r2 = enc(reinterpret_cast<CUtensorMap*>(ctx->tmap_a_rows), dt, 2, ctx->store, dims,
                      strides, box_row, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r2 != CUDA_SUCCESS)
        return dc_fail(ctx, DC_ERR_CUDA, "cuTensorMapEncodeTiled (row gathers) failed");
    for (int l = 0; l < ctx->cfg.levels * (ctx->lo_rows > 0 ? 2 : 1); l++) {
        const bool lo = l >= ctx->cfg.levels;  // FP32X3: maps of the lo copy
        const int lv = lo ? l - ctx->cfg.levels : l;
        const LevelBox lb = level_box(ctx, lv);
        cuuint64_t d4[4] = {(cuuint64_t)ctx->cfg.channels, (cuuint64_t)ctx->W[lv],
                            (cuuint64_t)ctx->H[lv], (cuuint64_t)ctx->cfg.max_frames};
        cuuint64_t s4[3] = {(cuuint64_t)row_bytes, (cuuint64_t)ctx->W[lv] * row_bytes,
                            (cuuint64_t)ctx->frame_rows * row_bytes};
        cuuint32_t b4[4] = {64, (cuuint32_t)lb.wbox, (cuuint32_t)lb.br, 1};
        cuuint32_t e4[4] = {1, 1, 1, 1};
        void* base = static_cast<char*>(ctx->store) +
                     (ctx->level_row0[lv] + (lo ? ctx->lo_rows : 0)) * row_bytes;
        unsigned char* tm = lo ? ctx->tmap_b_lo[lv] : ctx->tmap_b[lv];
        CUresult r = enc(reinterpret_cast<CUtensorMap*>(tm), dt, 4, base, d4, s4, b4,
                         e4, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS)
            return dc_fail(ctx, DC_ERR_CUDA, "cuTensorMapEncodeTiled (level rows) failed");
    }
    ctx->tc_ready = true;
    return DC_OK;
}

int dc_launch_tc(dc_ctx* ctx, const int* ii, const int* jj, int M, const float* coords,
                 float* out, cudaStream_t s) {
    if (!ctx->tc_ready) return dc_fail(ctx, DC_ERR_NOT_READY, "tensor maps not prepared");
    TcParams P;
    P.g = dc::geom_of(ctx);
    for (int l = 0; l < DC_MAX_LEVELS; l++)
        P.box[l] = l < ctx->cfg.levels ? level_box(ctx, l) : LevelBox{8, 1, 1, 0.125f};
    P.ii = ii;
    P.jj = jj;
    P.max_frames = ctx->cfg.max_frames;
    P.coords = coords;
    P.perm = nullptr;
    P.pflag = nullptr;
    P.pcoords = nullptr;
    P.out = out;
    P.err = ctx->dev_err;
    P.atoms = ctx->cfg.channels * 2 / 128;
    P.ab_fmt = ctx->cfg.precision == DC_PREC_BF16 ? 1u : 0u;
    P.M = M;
    // the short limit only ever comes with the stall: then no barrier phase the
    // epilogue warps wait on completes, so they all give up at the same chunk
    const long long lim = g_test_wait_ns.load();
    P.stall = lim > 0;
    P.wait_ns = lim > 0 ? (unsigned long long)lim : 2000000000ull;
    const int nkeys = ctx->H[0] + 2 * kBinPad;
    if (ctx->tile_order != DC_ORDER_SOURCE && ctx->tile_perm && M > 0 && nkeys <= kBinMaxKeys) {
        const size_t me = (size_t)ctx->cfg.max_edges, nhw = (size_t)ctx->hw;
        P.perm = ctx->tile_perm;
        P.pflag = ctx->tile_perm + me * nhw;
        P.pcoords = reinterpret_cast<const float*>(ctx->tile_perm + me * nhw + me);
        const int bsm = nkeys * 32 * (int)sizeof(int);
        cudaFuncSetAttribute(tile_order_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bsm);
        const int nch_o = ctx->cfg.levels * (2 * ctx->cfg.radius + 1) * (2 * ctx->cfg.radius + 1);
        tile_order_kernel<<<M, kBinThreads, bsm, s>>>(coords, ctx->hw, ctx->H[0], ctx->W[0],
                                                      nch_o, ctx->cfg.radius,
                                                      ctx->tile_order, ctx->tile_perm,
                                                      ctx->tile_perm + me * nhw,
                                                      const_cast<float*>(P.pcoords));
        const int rcb = dc_check_launch(ctx, "tile_order_kernel");
        if (rcb) return rcb;
    }
    const Layout Ly = make_layout(P.atoms);
    const size_t smem = Ly.total + 1024;
    const int ntiles = (ctx->hw + kTileM - 1) / kTileM * M;
    const int ctas = ctx->max_ctas > 0 && ctx->max_ctas < ctx->num_sms ? ctx->max_ctas : ctx->num_sms;
    dim3 grid(ntiles < ctas ? ntiles : ctas);
    // FP32X3: three passes, hi.hi + hi.lo + lo.hi, the later two adding to `out`
    const int passes = ctx->lo_rows > 0 ? 3 : 1;
    for (int pass = 0; pass < passes; pass++) {
        const bool a_lo = pass == 2, b_lo = pass == 1;
        P.a_off = a_lo ? ctx->lo_rows : 0;
        P.accum = pass > 0;
        P.keep = pass + 1 < passes;
        TcMaps maps;
        memset(&maps, 0, sizeof(maps));
        memcpy(&maps.a, ctx->tmap_a, sizeof(CUtensorMap));
        memcpy(&maps.a_rows, ctx->tmap_a_rows, sizeof(CUtensorMap));
        for (int l = 0; l < ctx->cfg.levels; l++)
            memcpy(&maps.b[l], b_lo ? ctx->tmap_b_lo[l] : ctx->tmap_b[l], sizeof(CUtensorMap));
#define DC_TC_LAUNCH(RR)                                                                 \
    do {                                                                                 \
        auto k = passes > 1 ? corr_tc_kernel<RR, true> : corr_tc_kernel<RR, false>;     \
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
        k<<<grid, kThreads, smem, s>>>(maps, P);                                         \
    } while (0)
        switch (ctx->cfg.radius) {
            case 0: DC_TC_LAUNCH(0); break;
            case 1: DC_TC_LAUNCH(1); break;
            case 2: DC_TC_LAUNCH(2); break;
            default: DC_TC_LAUNCH(3); break;
        }
#undef DC_TC_LAUNCH
        const int rc = dc_check_launch(ctx, "corr_tc_kernel");
        if (rc) return rc;
    }
    if (P.perm) {
        const int nch = ctx->cfg.levels * (2 * ctx->cfg.radius + 1) * (2 * ctx->cfg.radius + 1);
        const int usm = ctx->hw * (int)sizeof(float);
        cudaFuncSetAttribute(unpermute_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, usm);
        const dim3 ugrid(M, (nch + kUnpermRows - 1) / kUnpermRows);
        unpermute_rows_kernel<<<ugrid, kUnpermThreads, usm, s>>>(out, nch, ctx->hw, P.perm, P.pflag);
        const int rc = dc_check_launch(ctx, "unpermute_rows_kernel");
        if (rc) return rc;
    }
    return DC_OK;
}

// dc_tcvol.cu -- materialised level-0 volume on the tensor cores.
//
// The cublasGemmBatchedEx of cuda_slam/main.cu:1573-1581 (FP16 fmaps, fp32
// compute, V0[e][p][q] = alpha * sum_c f_ii[c][p] f_jj[c][q], row-major
// [source p][target q]) as tcgen05.mma: one CTA computes a 128 (p) x 256 (q)
// tile of one edge from the pixel-major store (K-major operands loaded by TMA,
// 128-byte swizzle), accumulates in TMEM (fp32), and four epilogue warps scale
// by alpha and store the tile with coalesced 512-byte row segments, staged
// through shared memory.  At fp32 output the build is HBM-store bound (about 60
// flop per byte), so one tile per CTA and two CTAs per SM keep the stores busy.
// Every wait is bounded (2 s) and reports through the context's error word.
#include <cuda.h>

#include "dc_internal.cuh"
#include "dc_sm100.cuh"

namespace {

using namespace dc::sm100;

constexpr int kTM = 128;          // source pixels per tile (MMA M, TMEM lanes)
constexpr int kTN = 256;          // target pixels per tile (MMA N, TMEM columns)
constexpr int kThreadsV = 192;    // warp 0: TMA + MMA, warp 1: TMEM allocator, 2..5: epilogue
constexpr uint32_t kRow = 128;    // bytes of one 64-element K atom row
constexpr int kStage = 36;        // floats per staged row (32 + pad)

struct VolParams {
    const int* ii;
    const int* jj;
    int max_frames;
    long long frame_rows;
    int hw;
    float alpha;
    float* vol0;
    int* err;
    int atoms;
    uint32_t ab_fmt;
    int tiles_p, tiles_q;
};

__global__ void __launch_bounds__(kThreadsV, 2)
    volume_tc_kernel(const __grid_constant__ CUtensorMap tmap, VolParams P) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base by pointer arithmetic on the shared array itself, so
    // that the compiler keeps the shared address space (LDS/STS, not generic)
    uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.y;
    const int tp = blockIdx.x / P.tiles_q, tq = blockIdx.x % P.tiles_q;
    const int p0 = tp * kTM, q0 = tq * kTN;
    const int si = P.ii[e], sj = P.jj[e];
    const int hw = P.hw;
    float* V = P.vol0 + (size_t)e * hw * hw;
    if (!(si >= 0 && si < P.max_frames && sj >= 0 && sj < P.max_frames)) {
        for (int idx = threadIdx.x; idx < kTM * kTN; idx += kThreadsV) {
            const int p = p0 + idx / kTN, q = q0 + idx % kTN;
            if (p < hw && q < hw) V[(size_t)p * hw + q] = 0.0f;
        }
        return;
    }
    const uint32_t sA = smem_addr(base);
    const uint32_t sB = sA + P.atoms * kTM * kRow;
    // the epilogue's staging rows reuse the operand tiles (free once the MMAs completed)
    float* stage = reinterpret_cast<float*>(base);
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + P.atoms * (kTM + kTN) * kRow);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tslot + 1);
    const uint32_t bar_in = smem_addr(&bars[0]), bar_mma = smem_addr(&bars[1]);

    if (threadIdx.x == 0) {
        mbar_init(bar_in, 1);
        mbar_init(bar_mma, 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tslot), kTN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == 0) {
        if (lane == 0) {
            mbar_arrive_expect_tx(bar_in, P.atoms * (kTM + kTN) * kRow);
            const int arow = (int)((long long)si * P.frame_rows + p0);
            const int brow = (int)((long long)sj * P.frame_rows + q0);
            for (int k = 0; k < P.atoms; k++) {
                tma_load_2d(sA + k * kTM * kRow, &tmap, k * 64, arow, bar_in);
                for (int h = 0; h < kTN / 128; h++)
                    tma_load_2d(sB + k * kTN * kRow + h * 128 * kRow, &tmap, k * 64,
                                brow + h * 128, bar_in);
            }
            if (!mbar_wait(bar_in, 0, abort)) {
                *abort = 1;
                atomicExch(P.err, 11);
                mma_commit(bar_mma);  // releases the epilogue (no MMA was issued)
            } else {
                tc_fence_after();
                const uint32_t idesc = idesc_f16(P.ab_fmt, kTM, kTN);
                for (int kk = 0; kk < P.atoms * 4; kk++) {
                    const int at = kk >> 2, wi = kk & 3;
                    mma_f16(tmem, sdesc_sw128(sA + at * kTM * kRow + wi * 32),
                            sdesc_sw128(sB + at * kTN * kRow + wi * 32), idesc, kk > 0);
                }
                mma_commit(bar_mma);
            }
        }
        __syncwarp();
    } else if (warp >= 2) {
        // epilogue: warp w reads TMEM lanes 32*(w%4).. = tile rows; 32 columns at
        // a time, staged so that each store instruction writes whole row segments
        const int quarter = warp & 3;
        float* st = stage + (warp - 2) * 32 * kStage;
        int ok = 1;
        if (lane == 0) ok = mbar_wait(bar_mma, 0, abort) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (ok && !*abort) {
            mbar_wait(bar_mma, 0, abort);
            tc_fence_after();
            const uint32_t tl = tmem + ((uint32_t)(32 * quarter) << 16);
            for (int cb = 0; cb < kTN; cb += 32) {
                float v[32];
                tmem_ld32(tl + (uint32_t)cb, v);
                __syncwarp();
#pragma unroll
                for (int k = 0; k < 8; k++)
                    *reinterpret_cast<float4*>(st + lane * kStage + 4 * k) =
                        make_float4(P.alpha * v[4 * k], P.alpha * v[4 * k + 1],
                                    P.alpha * v[4 * k + 2], P.alpha * v[4 * k + 3]);
                __syncwarp();
                // lanes 8r..8r+7 store row (4 * it + r), 16 bytes each
                const int q = q0 + cb + 4 * (lane & 7);
#pragma unroll
                for (int it = 0; it < 8; it++) {
                    const int rr = 4 * it + (lane >> 3);
                    const int p = p0 + 32 * quarter + rr;
                    if (p >= hw) continue;
                    const float4 val = *reinterpret_cast<const float4*>(st + rr * kStage + 4 * (lane & 7));
                    float* dst = V + (size_t)p * hw + q;
                    if (q + 3 < hw && (hw & 3) == 0) {
                        __stcs(reinterpret_cast<float4*>(dst), val);
                    } else {
                        if (q < hw) dst[0] = val.x;
                        if (q + 1 < hw) dst[1] = val.y;
                        if (q + 2 < hw) dst[2] = val.z;
                        if (q + 3 < hw) dst[3] = val.w;
                    }
                }
            }
        } else if (lane == 0) {
            atomicExch(P.err, 12);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTN);
    }
}

}  // namespace

int dc_launch_volume_tc(dc_ctx* ctx, const int* ii, const int* jj, int M, float* vol0,
                        cudaStream_t s) {
    if (!ctx->tc_ready) return dc_fail(ctx, DC_ERR_NOT_READY, "tensor maps not prepared");
    VolParams P;
    P.ii = ii;
    P.jj = jj;
    P.max_frames = ctx->cfg.max_frames;
    P.frame_rows = ctx->frame_rows;
    P.hw = ctx->hw;
    P.alpha = ctx->cfg.alpha;
    P.vol0 = vol0;
    P.err = ctx->dev_err;
    P.atoms = ctx->cfg.channels * 2 / 128;
    P.ab_fmt = ctx->cfg.precision == DC_PREC_BF16 ? 1u : 0u;
    P.tiles_p = (ctx->hw + kTM - 1) / kTM;
    P.tiles_q = (ctx->hw + kTN - 1) / kTN;
    const size_t smem = 1024 + (size_t)P.atoms * (kTM + kTN) * kRow + 64;
    static_assert(4 * 32 * kStage * sizeof(float) <= 1 * (kTM + kTN) * kRow, "staging fits");
    cudaFuncSetAttribute(volume_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    dim3 grid(P.tiles_p * P.tiles_q, M);
    volume_tc_kernel<<<grid, kThreadsV, smem, s>>>(
        *reinterpret_cast<const CUtensorMap*>(ctx->tmap_a), P);
    return dc_check_launch(ctx, "volume_tc_kernel");
}

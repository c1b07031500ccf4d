// dc_enc.cu -- the update operator's correlation encoder, first layer, on the
// tensor cores: out = fp16(relu(W corr + b)), a 1x1 convolution from the
// lookup's levels*(2r+1)^2 = 196 channels to 128.
//
// Replaces UpdateModule's corr_enc_0 (cuDNN 1x1 convolution, 196 -> 128, with
// bias; cuda_slam/main.cu:552-553) followed by relu_inplace and round_to_fp16
// (main.cu:603-606), which read the 196-channel fp32 correlation features and
// write 128 fp32 channels holding fp16-rounded values.  Here the result is
// written as fp16 (the same values, half the bytes).
//
// Per tile of 128 pixels of one edge (persistent CTAs, 512 threads): four
// threads per pixel each read a quarter of its 196 features (coalesced along
// pixels, 64 loads in flight per thread), round them to fp16 and write them to
// shared memory as the K-major A operand (128-byte swizzle, K padded with
// zeros to 256); the weights, packed once by dc_set_corr_encoder
// into the same layout, stay resident in shared memory as the B operand; one
// thread issues 16 tcgen05.mma (kind::f16, M = N = 128, K = 16) into a TMEM
// accumulator; each warp reads 32 outputs of its lane quarter's 32 pixels back
// (tcgen05.ld), adds the bias, applies the ReLU, rounds to fp16 and stores
// 64-byte rows.
// That kernel serves grids whose h*w is not a multiple of 8 or is below 128;
// for the others corr_encoder_tma_kernel streams the features with TMA
// (below).
// The waits for the MMAs and the boxes are bounded (2 s) and report through
// the context's device error word.
#include <cuda.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <cstring>

#include "dc_internal.cuh"
#include "dc_sm100.cuh"

namespace {

using namespace dc::sm100;

constexpr int kEncM = 128;        // pixels per tile (MMA M, TMEM lanes)
constexpr int kEncCo = 128;       // output channels (MMA N)
constexpr int kEncK = 256;        // input channels, padded (four 64-element K atoms)
constexpr int kEncThreads = 512;  // 4 threads per pixel row of the tile
constexpr int kEncParts = kEncThreads / kEncM;
constexpr uint32_t kAtomBytes = 128u * 128u;            // 128 rows x 128 bytes
constexpr uint32_t kOperandBytes = 4u * kAtomBytes;     // 64 KB
constexpr uint32_t kWeightBytes = kOperandBytes;

// Byte offset of element (row r, k) in the 128-byte-swizzled K-major layout:
// K atom k / 64, row r at 128 bytes, 16-byte chunk (k % 64) / 8 stored at
// chunk ^ (r % 8).
__host__ __device__ __forceinline__ uint32_t sw128_offset(int r, int k) {
    const int atom = k >> 6, kk = k & 63;
    return (uint32_t)atom * kAtomBytes + (uint32_t)r * 128u +
           (uint32_t)((((kk >> 3) ^ (r & 7)) << 4) | ((kk & 7) << 1));
}

__global__ void enc_pack_weights_kernel(const float* __restrict__ w, int ci,
                                        __half* __restrict__ img) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;  // co * kEncK + k
    if (idx >= kEncCo * kEncK) return;
    const int co = idx / kEncK, k = idx % kEncK;
    const float v = k < ci ? w[co * ci + k] : 0.0f;
    img[sw128_offset(co, k) / 2] = __float2half_rn(v);
}

struct EncParams {
    const float* corr;  // [M][ci][hw]
    const uint4* wimg;  // packed weights (kWeightBytes)
    const float* bias;  // [128]
    __half* out;        // [M][128][hw]
    int* err;
    int M, ci, hw;
};

__global__ void __launch_bounds__(kEncThreads, 1) corr_encoder_kernel(EncParams P) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint8_t* sB = base;                    // weights
    uint8_t* sA = base + kWeightBytes;     // pixel tile
    uint64_t* bar = reinterpret_cast<uint64_t*>(sA + kOperandBytes);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hw = P.hw;
    const int tpe = (hw + kEncM - 1) / kEncM;
    const int ntiles = tpe * P.M;

    // resident weights (L2 -> shared, 16-byte loads)
    for (int i = tid; i < (int)(kWeightBytes / 16); i += kEncThreads)
        reinterpret_cast<uint4*>(sB)[i] = __ldg(P.wimg + i);
    if (tid == 0) {
        mbar_init(smem_addr(bar), 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_addr(tslot), 128);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t idesc = idesc_f16(0u, kEncM, kEncCo);
    const uint32_t aA = smem_addr(sA), aB = smem_addr(sB);
    int phase = 0;
    bool alive = true;

    for (int t = blockIdx.x; t < ntiles && alive; t += gridDim.x, phase ^= 1) {
        const int e = t / tpe, p0 = (t - e * tpe) * kEncM;
        const int row = tid % kEncM, part = tid / kEncM;
        const int p = p0 + row;
        const bool pv = p < hw;
        // A tile: row = pixel p, 8 channels per 16-byte chunk; this thread's
        // quarter of the chunks, all loads issued before any is used
        const float* src = P.corr + (size_t)e * P.ci * hw + p;
#pragma unroll
        for (int cc = 0; cc < kEncK / 8 / kEncParts; cc++) {
            const int c = part * (kEncK / 8 / kEncParts) + cc;
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int k = 8 * c + j;
                v[j] = (pv && k < P.ci) ? __ldcs(src + (size_t)k * hw) : 0.0f;
            }
            uint4 pk;
            __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
            __half2 h2 = __floats2half2_rn(v[4], v[5]), h3 = __floats2half2_rn(v[6], v[7]);
            pk.x = *reinterpret_cast<uint32_t*>(&h0);
            pk.y = *reinterpret_cast<uint32_t*>(&h1);
            pk.z = *reinterpret_cast<uint32_t*>(&h2);
            pk.w = *reinterpret_cast<uint32_t*>(&h3);
            *reinterpret_cast<uint4*>(sA + sw128_offset(row, 8 * c)) = pk;
        }
        fence_proxy_async();  // generic-proxy stores -> tensor-core reads
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < kEncK / 16; kk++) {
                const int at = kk >> 2, wi = kk & 3;
                mma_f16(tmem, sdesc_sw128(aA + at * kAtomBytes + wi * 32),
                        sdesc_sw128(aB + at * kAtomBytes + wi * 32), idesc, kk > 0 ? 1u : 0u);
            }
            mma_commit(smem_addr(bar));
        }
        __syncwarp();
        int ok = 1;
        if (lane == 0) ok = mbar_wait(smem_addr(bar), phase, nullptr) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (ok) mbar_wait(smem_addr(bar), phase, nullptr);
        if (!ok) {
            if (lane == 0) atomicExch(P.err, 20);
            alive = false;
        }
        // every warp must reach the barrier below, whether or not it gave up
        if (alive) {
            // warp w: TMEM lane quarter w % 4 (pixels 32 (w % 4) ..), output
            // channels 32 (w / 4) .. 32 (w / 4) + 31
            tc_fence_after();
            const int q = warp & 3, cb = 32 * (warp >> 2);
            const int pq = p0 + 32 * q + lane;
            const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16) + cb;
            float acc[32];
            tmem_ld32(tl, acc);
            if (pq < hw) {
                __half* o = P.out + (size_t)e * kEncCo * hw + pq;
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    const int co = cb + j;
                    const float y = fmaxf(acc[j] + __ldg(P.bias + co), 0.0f);
                    o[(size_t)co * hw] = __float2half_rn(y);
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        // a warp that timed out leaves the loop; so do the others (bar.sync
        // above has collected every warp; the flag is re-read uniformly)
        alive = __syncthreads_and(alive ? 1 : 0) != 0;
    }
    if (!alive && tid == 0) {
        // the MMAs of the abandoned tile may still read shared memory: wait (bounded)
        mbar_wait(smem_addr(bar), phase, nullptr);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 128);
    }
}

// The same layer with the feature tile streamed by TMA (h*w a multiple of 8,
// features 16-byte aligned): one thread keeps kEncStages boxes of 64 channels
// x 128 pixels fp32 (32 KB) in flight in a shared-memory ring, so the next
// tile's loads overlap this tile's conversion, MMAs and stores.  All threads
// convert a landed box into the fp16 K-major operand (4 threads per pixel row,
// one 16-byte chunk of 8 channels each per pass); the last box of a tile holds
// the remaining channels rounded up to 16 (rows past the channels, which
// belong to the next edge or lie outside the tensor, are written as zeros).
// Only the K steps that hold channels are issued.  Outputs are staged as fp16
// [co][128 pixels] in the consumed operand tile and stored as 16-byte runs.
constexpr int kEncStages = 3;
constexpr uint32_t kStageBytes = 64u * kEncM * 4u;

struct EncTmaParams {
    const uint4* wimg;
    const float* bias;
    __half* out;
    int* err;
    int M, ci, hw;
    int nfull;      // 64-channel boxes per tile
    int tail_rows;  // channels of the last box, a multiple of 16 (0: none)
};

__global__ void __launch_bounds__(kEncThreads, 1)
    corr_encoder_tma_kernel(const __grid_constant__ CUtensorMap mfull,
                            const __grid_constant__ CUtensorMap mtail, EncTmaParams P) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint8_t* sB = base;                          // weights
    uint8_t* sA = base + kWeightBytes;           // fp16 pixel tile / output staging
    uint8_t* ring = sA + kOperandBytes;          // kEncStages fp32 boxes
    uint64_t* bars = reinterpret_cast<uint64_t*>(ring + kEncStages * kStageBytes);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + kEncStages + 1);
    float* sbias = reinterpret_cast<float*>(ring + kEncStages * kStageBytes + 64);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hw = P.hw;
    const int tpe = (hw + kEncM - 1) / kEncM;
    const int ntiles = tpe * P.M;
    const int cpt = P.nfull + (P.tail_rows > 0 ? 1 : 0);  // boxes per tile
    const int my_tiles = (int)blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nchunks = my_tiles * cpt;
    const uint32_t mma_bar = smem_addr(bars + kEncStages);
    const int ksteps = (P.ci + 15) / 16;

    for (int i = tid; i < (int)(kWeightBytes / 16); i += kEncThreads)
        reinterpret_cast<uint4*>(sB)[i] = __ldg(P.wimg + i);
    if (tid < kEncCo) sbias[tid] = __ldg(P.bias + tid);
    if (tid == 0) {
        for (int st = 0; st <= kEncStages; st++) mbar_init(smem_addr(bars + st), 1);
        fence_mbar_init();
        tma_prefetch_desc(&mfull);
        tma_prefetch_desc(&mtail);
    }
    if (warp == 0) {
        tmem_alloc(smem_addr(tslot), 128);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t idesc = idesc_f16(0u, kEncM, kEncCo);
    const uint32_t aA = smem_addr(sA), aB = smem_addr(sB);

    // box g of this CTA: tile blockIdx.x + (g / cpt) * gridDim.x, box g % cpt
    int issued = 0;  // (thread 0)
    auto issue = [&](int gi) {
        const int t = (int)blockIdx.x + (gi / cpt) * (int)gridDim.x, c = gi % cpt;
        const int e = t / tpe, p0 = (t - e * tpe) * kEncM;
        const int st = gi % kEncStages;
        const bool tail = c == P.nfull;
        mbar_arrive_expect_tx(smem_addr(bars + st), (tail ? P.tail_rows : 64) * kEncM * 4u);
        tma_load_2d(smem_addr(ring + st * kStageBytes), tail ? (const void*)&mtail : (const void*)&mfull,
                    p0, e * P.ci + 64 * c, smem_addr(bars + st));
        issued = gi + 1;
    };
    if (tid == 0)
        for (int gi = 0; gi < min(kEncStages, nchunks); gi++) issue(gi);

    int g = 0, mphase = 0;
    bool alive = true, mma_out = false;
    for (int t = blockIdx.x; t < ntiles && alive; t += gridDim.x, mphase ^= 1) {
        const int e = t / tpe, p0 = (t - e * tpe) * kEncM;
        for (int c = 0; c < cpt; c++, g++) {
            const int st = g % kEncStages;
            int ok = 1;
            if (lane == 0) ok = mbar_wait(smem_addr(bars + st), (g / kEncStages) & 1, nullptr) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (ok) {
                mbar_wait(smem_addr(bars + st), (g / kEncStages) & 1, nullptr);
                const float* box = reinterpret_cast<const float*>(ring + st * kStageBytes);
                const int rows = c == P.nfull ? P.tail_rows : 64;
                const int px = tid & (kEncM - 1), part = tid >> 7;
                for (int o = part; o < rows / 8; o += kEncParts) {
                    float f[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int k = 64 * c + 8 * o + j;
                        f[j] = k < P.ci ? box[(8 * o + j) * kEncM + px] : 0.0f;
                    }
                    __half2 h0 = __floats2half2_rn(f[0], f[1]), h1 = __floats2half2_rn(f[2], f[3]);
                    __half2 h2 = __floats2half2_rn(f[4], f[5]), h3 = __floats2half2_rn(f[6], f[7]);
                    uint4 pk;
                    pk.x = *reinterpret_cast<uint32_t*>(&h0);
                    pk.y = *reinterpret_cast<uint32_t*>(&h1);
                    pk.z = *reinterpret_cast<uint32_t*>(&h2);
                    pk.w = *reinterpret_cast<uint32_t*>(&h3);
                    *reinterpret_cast<uint4*>(sA + sw128_offset(px, 64 * c + 8 * o)) = pk;
                }
                fence_proxy_async();  // generic-proxy stores -> tensor-core reads
            } else if (lane == 0) {
                atomicExch(P.err, 21);
            }
            // the box is consumed (or abandoned) by every thread: refill its slot
            alive = __syncthreads_and(ok) != 0;
            if (!alive) break;
            if (tid == 0 && g + kEncStages < nchunks) issue(g + kEncStages);
        }
        if (!alive) break;
        if (tid == 0) {
            tc_fence_after();
            for (int kk = 0; kk < ksteps; kk++) {
                const int at = kk >> 2, wi = kk & 3;
                mma_f16(tmem, sdesc_sw128(aA + at * kAtomBytes + wi * 32),
                        sdesc_sw128(aB + at * kAtomBytes + wi * 32), idesc, kk > 0 ? 1u : 0u);
            }
            mma_commit(mma_bar);
        }
        mma_out = true;
        int ok = 1;
        if (lane == 0) ok = mbar_wait(mma_bar, mphase, nullptr) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (ok) {
            mbar_wait(mma_bar, mphase, nullptr);
            mma_out = false;
            tc_fence_after();
            // warp w: TMEM lane quarter w % 4 (pixels 32 (w % 4) ..), output
            // channels 32 (w / 4) ..; staged as [co][128 pixels] fp16
            const int q = warp & 3, cb = 32 * (warp >> 2);
            float acc[32];
            tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + cb, acc);
            __half* stg = reinterpret_cast<__half*>(sA);
#pragma unroll
            for (int j = 0; j < 32; j++) {
                const int co = cb + j;
                stg[co * kEncM + 32 * q + lane] = __float2half_rn(fmaxf(acc[j] + sbias[co], 0.0f));
            }
        } else if (lane == 0) {
            atomicExch(P.err, 20);
        }
        tc_fence_before();
        alive = __syncthreads_and(ok) != 0;
        if (alive) {
            const uint4* stg = reinterpret_cast<const uint4*>(sA);
            __half* oe = P.out + (size_t)e * kEncCo * hw + p0;
#pragma unroll
            for (int j = 0; j < kEncCo * kEncM / 8 / kEncThreads; j++) {
                const int cc = tid + kEncThreads * j;  // co = cc / 16, 8 pixels each
                const int co = cc >> 4, x8 = (cc & 15) * 8;
                if (p0 + x8 < hw) __stcs(reinterpret_cast<uint4*>(oe + (size_t)co * hw + x8), stg[cc]);
            }
        }
        __syncthreads();  // the staged outputs are read before the next tile's operand
    }
    if (!alive && tid == 0) {
        // boxes still in flight and an abandoned MMA group: let them land (bounded)
        for (int gi = g; gi < issued; gi++)
            mbar_wait(smem_addr(bars + gi % kEncStages), (gi / kEncStages) & 1, nullptr);
        if (mma_out) mbar_wait(mma_bar, mphase, nullptr);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 128);
    }
}

}  // namespace

int dc_set_corr_encoder_impl(dc_ctx* ctx, const float* weight, const float* bias, int co,
                             cudaStream_t s) {
    const int ci = ctx->cfg.levels * (2 * ctx->cfg.radius + 1) * (2 * ctx->cfg.radius + 1);
    if (co != kEncCo)
        return dc_fail(ctx, DC_ERR_UNSUPPORTED, "the correlation encoder has 128 output channels");
    if (ci > kEncK)
        return dc_fail(ctx, DC_ERR_UNSUPPORTED, "more than 256 correlation channels");
    if (!ctx->enc_w) {
        if (cudaMalloc(&ctx->enc_w, kWeightBytes + kEncCo * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            ctx->enc_w = nullptr;
            return dc_fail(ctx, DC_ERR_NO_MEMORY, "encoder weights");
        }
        ctx->other_bytes += (long long)(kWeightBytes + kEncCo * sizeof(float));
    }
    float* b = reinterpret_cast<float*>(static_cast<char*>(ctx->enc_w) + kWeightBytes);
    enc_pack_weights_kernel<<<(kEncCo * kEncK + 255) / 256, 256, 0, s>>>(
        weight, ci, static_cast<__half*>(ctx->enc_w));
    int rc = dc_check_launch(ctx, "enc_pack_weights_kernel");
    if (rc) return rc;
    if (cudaMemcpyAsync(b, bias, kEncCo * sizeof(float), cudaMemcpyDeviceToDevice, s) !=
        cudaSuccess)
        return dc_fail(ctx, DC_ERR_CUDA, "copying the encoder bias failed");
    ctx->enc_ready = true;
    return DC_OK;
}

int dc_launch_encoder(dc_ctx* ctx, const float* corr, int M, void* out, cudaStream_t s) {
    if (!ctx->enc_ready)
        return dc_fail(ctx, DC_ERR_NOT_READY, "dc_set_corr_encoder has not been called");
    EncParams P;
    P.corr = corr;
    P.wimg = static_cast<const uint4*>(ctx->enc_w);
    P.bias = reinterpret_cast<const float*>(static_cast<char*>(ctx->enc_w) + kWeightBytes);
    P.out = static_cast<__half*>(out);
    P.err = ctx->dev_err;
    P.M = M;
    P.ci = ctx->cfg.levels * (2 * ctx->cfg.radius + 1) * (2 * ctx->cfg.radius + 1);
    P.hw = ctx->hw;
    const int ntiles = (ctx->hw + kEncM - 1) / kEncM * M;
    const int grid = ntiles < ctx->num_sms ? ntiles : ctx->num_sms;
    // TMA path: rows of whole 16-byte runs, aligned buffers, and at least one
    // full 128-pixel box per row
    if (ctx->hw % 8 == 0 && ctx->hw >= kEncM && ((uintptr_t)corr & 15) == 0 &&
        ((uintptr_t)out & 15) == 0) {
        EncTmaParams T;
        T.wimg = P.wimg;
        T.bias = P.bias;
        T.out = P.out;
        T.err = P.err;
        T.M = M;
        T.ci = P.ci;
        T.hw = P.hw;
        T.nfull = P.ci / 64;
        T.tail_rows = (P.ci - 64 * T.nfull + 15) / 16 * 16;
        alignas(64) unsigned char mf[128], mt[128];
        const unsigned long long rows = (unsigned long long)M * P.ci;
        if (dc_tmap_2d_f32(mf, corr, (unsigned long long)P.hw, rows, kEncM, 64) != DC_OK ||
            (T.tail_rows > 0 &&
             dc_tmap_2d_f32(mt, corr, (unsigned long long)P.hw, rows, kEncM, T.tail_rows) != DC_OK))
            return dc_fail(ctx, DC_ERR_CUDA, "cuTensorMapEncodeTiled (corr features) failed");
        if (T.tail_rows == 0) memcpy(mt, mf, sizeof(mt));
        const size_t tsmem = 2 * kOperandBytes + kEncStages * kStageBytes + 64 +
                             kEncCo * sizeof(float) + 1024;
        cudaFuncSetAttribute(corr_encoder_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)tsmem);
        corr_encoder_tma_kernel<<<grid, kEncThreads, tsmem, s>>>(
            *reinterpret_cast<const CUtensorMap*>(mf), *reinterpret_cast<const CUtensorMap*>(mt), T);
        return dc_check_launch(ctx, "corr_encoder_tma_kernel");
    }
    const size_t smem = 2 * kOperandBytes + 64 + 1024;
    cudaFuncSetAttribute(corr_encoder_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    corr_encoder_kernel<<<grid, kEncThreads, smem, s>>>(P);
    return dc_check_launch(ctx, "corr_encoder_kernel");
}

// dc_api.cu -- the C ABI of libdroidcorr: argument validation, the context and
// dispatch to the kernels.  Declarations and the reference interface each entry
// point replaces are in include/droidcorr.h.
#include <cstdio>
#include <cstring>

#include <cuda.h>

#include "dc_internal.cuh"

int dc_fail(dc_ctx* ctx, int status, const std::string& msg) {
    if (ctx) ctx->err = msg;
    return status;
}

int dc_check_launch(dc_ctx* ctx, const char* what) {
    ctx->launches++;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return dc_fail(ctx, DC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    return DC_OK;
}

namespace {

constexpr long long kSyncPageBytes = 4096;
constexpr int kSyncWords = (int)(kSyncPageBytes / 4);

typedef CUresult (*StreamValueFn)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

StreamValueFn stream_value_fn(const char* name) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
        return nullptr;
    return reinterpret_cast<StreamValueFn>(p);
}

// Word `word` of this context's counter page, or of the attached source's.
CUdeviceptr sync_word(const dc_ctx* ctx, int word, bool remote) {
    const char* base = static_cast<const char*>(remote ? ctx->src_store : ctx->store);
    return reinterpret_cast<CUdeviceptr>(base + ctx->store_bytes + 4LL * word);
}

int validate_edges(dc_ctx* ctx, const int* ii, const int* jj, int M) {
    if (M < 0 || M > ctx->cfg.max_edges)
        return dc_fail(ctx, DC_ERR_INVALID_ARG,
                       "M=" + std::to_string(M) + " outside [0, max_edges=" +
                           std::to_string(ctx->cfg.max_edges) + "]");
    if (M > 0 && (!ii || !jj)) return dc_fail(ctx, DC_ERR_INVALID_ARG, "ii/jj is NULL");
    return DC_OK;
}

}  // namespace

int dc_init_geometry(dc_ctx* ctx, const dc_config& c, int frames) {
    if (c.h < 1 || c.w < 1 || (long long)c.h * c.w > DC_MAX_HW) return DC_ERR_INVALID_ARG;
    if (c.channels != 32 && c.channels != 64 && c.channels != 128 && c.channels != 256)
        return DC_ERR_INVALID_ARG;
    if (c.levels < 1 || c.levels > DC_MAX_LEVELS) return DC_ERR_INVALID_ARG;
    if (c.radius < 0 || c.radius > DC_MAX_RADIUS) return DC_ERR_INVALID_ARG;
    if (c.precision < DC_PREC_FP32 || c.precision > DC_PREC_FP32X3) return DC_ERR_INVALID_ARG;
    if (c.precision == DC_PREC_FP32X3 && c.channels != 64 && c.channels != 128)
        return DC_ERR_INVALID_ARG;
    if ((c.h >> (c.levels - 1)) < 1 || (c.w >> (c.levels - 1)) < 1) return DC_ERR_INVALID_ARG;
    ctx->cfg = c;
    ctx->hw = c.h * c.w;
    long long rows = 0;
    for (int l = 0; l < DC_MAX_LEVELS; l++) {
        ctx->H[l] = c.h >> l;
        ctx->W[l] = c.w >> l;
        ctx->level_row0[l] = rows;
        if (l < c.levels) {
            long long n = (long long)ctx->H[l] * ctx->W[l];
            rows += (n + DC_ROW_PAD - 1) / DC_ROW_PAD * DC_ROW_PAD;
        }
    }
    // FP32X3 keeps a lo copy of every slot right after its hi rows
    ctx->lo_rows = c.precision == DC_PREC_FP32X3 ? rows : 0;
    ctx->frame_rows = c.precision == DC_PREC_FP32X3 ? 2 * rows : rows;
    ctx->elem_bytes = dc_store_is_16bit(c.precision) ? 2 : 4;
    ctx->store_bytes = (long long)frames * ctx->frame_rows * c.channels * ctx->elem_bytes;
    return DC_OK;
}

extern "C" {

void dc_default_config(dc_config* cfg, int h, int w) {
    cfg->h = h;
    cfg->w = w;
    cfg->channels = 128;
    cfg->levels = 4;
    cfg->radius = 3;
    cfg->max_frames = 512;
    cfg->max_edges = 48;
    cfg->precision = DC_PREC_FP16;
    cfg->alpha = 1.0f / 16.0f;
}

const char* dc_status_string(int s) {
    switch (s) {
        case DC_OK: return "ok";
        case DC_ERR_INVALID_ARG: return "invalid argument";
        case DC_ERR_CUDA: return "CUDA error";
        case DC_ERR_UNSUPPORTED: return "unsupported configuration";
        case DC_ERR_NO_MEMORY: return "out of device memory";
        case DC_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
        case DC_ERR_NOT_READY: return "not ready";
        default: return "unknown status";
    }
}

int dc_create(const dc_config* cfg, dc_ctx** out) {
    if (!cfg || !out) return DC_ERR_INVALID_ARG;
    *out = nullptr;
    const dc_config& c = *cfg;
    if (c.max_frames < 1 || c.max_edges < 1) return DC_ERR_INVALID_ARG;
    dc_ctx* ctx = new dc_ctx();
    if (dc_init_geometry(ctx, c, c.max_frames) != DC_OK) {
        delete ctx;
        return DC_ERR_INVALID_ARG;
    }
    if (cudaGetDevice(&ctx->device) != cudaSuccess) {
        delete ctx;
        return DC_ERR_CUDA;
    }
    cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, ctx->device);
    // the store, then one 4 KB page of replication counters (dc_sync_signal)
    if (cudaMalloc(&ctx->store, ctx->store_bytes + kSyncPageBytes) != cudaSuccess) {
        cudaGetLastError();
        delete ctx;
        return DC_ERR_NO_MEMORY;
    }
    // Padding rows must read as zero; the store is written slot by slot later.
    if (cudaMemset(ctx->store, 0, ctx->store_bytes + kSyncPageBytes) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(ctx->store);
        delete ctx;
        return DC_ERR_CUDA;
    }
    // one small allocation: the device error word, then the scatter-mean lists
    // (dc_scatter_mean: edge order, list offsets and mean scales, max_edges each)
    const size_t small_words = 32 + 3 * (size_t)c.max_edges + 1;
    ctx->other_bytes += (long long)(small_words * sizeof(int));
    if (cudaMalloc(&ctx->dev_err, small_words * sizeof(int)) != cudaSuccess ||
        cudaMemset(ctx->dev_err, 0, sizeof(int)) != cudaSuccess) {
        cudaFree(ctx->store);
        delete ctx;
        return DC_ERR_NO_MEMORY;
    }
    if (dc_tc_supported(ctx)) {
        int rc = dc_tc_prepare(ctx);
        if (rc != DC_OK) {
            cudaFree(ctx->dev_err);
            cudaFree(ctx->store);
            delete ctx;
            return rc;
        }
    }
    cudaDeviceSynchronize();
    *out = ctx;
    return DC_OK;
}

int dc_destroy(dc_ctx* ctx) {
    if (!ctx) return DC_OK;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(ctx->device);
    if (ctx->store) cudaFree(ctx->store);
    if (ctx->dev_err) cudaFree(ctx->dev_err);
    if (ctx->enc_w) cudaFree(ctx->enc_w);
    if (ctx->tile_perm) cudaFree(ctx->tile_perm);
    if (ctx->src_store) cudaIpcCloseMemHandle(ctx->src_store);
    if (prev >= 0) cudaSetDevice(prev);
    delete ctx;
    return DC_OK;
}

const char* dc_last_error(const dc_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

long long dc_context_bytes(const dc_ctx* ctx) {
    return ctx ? ctx->store_bytes + kSyncPageBytes + ctx->other_bytes : 0;
}

long long dc_launch_count(const dc_ctx* ctx) { return ctx ? ctx->launches : 0; }

int dc_set_max_ctas(dc_ctx* ctx, int max_ctas) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    if (max_ctas < 0) return dc_fail(ctx, DC_ERR_INVALID_ARG, "max_ctas < 0");
    ctx->max_ctas = max_ctas;
    return DC_OK;
}

int dc_set_tile_order(dc_ctx* ctx, int order) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    if (order != DC_ORDER_SOURCE && order != DC_ORDER_WINDOW_ROW && order != DC_ORDER_AUTO)
        return dc_fail(ctx, DC_ERR_INVALID_ARG, "order must be DC_ORDER_SOURCE, _WINDOW_ROW or _AUTO");
    if (order != DC_ORDER_SOURCE && !ctx->tile_perm) {
        // per edge: the permutation (hw), its flag (1), the permuted coordinates (2 hw)
        const size_t words = (size_t)ctx->cfg.max_edges * (3 * (size_t)ctx->hw + 1);
        int prev = -1;
        cudaGetDevice(&prev);
        cudaSetDevice(ctx->device);
        const cudaError_t e = cudaMalloc(&ctx->tile_perm, words * sizeof(int));
        if (prev >= 0) cudaSetDevice(prev);
        if (e != cudaSuccess) {
            ctx->tile_perm = nullptr;
            cudaGetLastError();
            return dc_fail(ctx, DC_ERR_NO_MEMORY, "tile permutation scratch");
        }
        ctx->other_bytes += (long long)(words * sizeof(int));
    }
    ctx->tile_order = order;
    return DC_OK;
}

int dc_set_frames(dc_ctx* ctx, const void* fmaps, int dtype, int first, int count,
                  dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    if (dtype != DC_DTYPE_F32 && dtype != DC_DTYPE_F16)
        return dc_fail(ctx, DC_ERR_INVALID_ARG, "dtype must be DC_DTYPE_F32 or DC_DTYPE_F16");
    if (first < 0 || count < 0 || first + count > ctx->cfg.max_frames)
        return dc_fail(ctx, DC_ERR_INVALID_ARG, "slot range outside [0, max_frames)");
    if (count == 0) return DC_OK;
    if (!fmaps) return dc_fail(ctx, DC_ERR_INVALID_ARG, "fmaps is NULL");
    return dc_launch_store(ctx, fmaps, dtype, first, count, (cudaStream_t)stream);
}

int dc_store_slots(dc_ctx* ctx, int first, int count, void** ptr, long long* bytes) {
    if (!ctx || !ptr || !bytes) return DC_ERR_INVALID_ARG;
    if (first < 0 || count < 0 || first + count > ctx->cfg.max_frames)
        return dc_fail(ctx, DC_ERR_INVALID_ARG, "slot range outside [0, max_frames)");
    const long long slot_bytes = ctx->frame_rows * ctx->cfg.channels * ctx->elem_bytes;
    *ptr = static_cast<char*>(ctx->store) + first * slot_bytes;
    *bytes = count * slot_bytes;
    return DC_OK;
}

int dc_store_ipc_handle(dc_ctx* ctx, void* handle_out) {
    if (!ctx || !handle_out) return DC_ERR_INVALID_ARG;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, ctx->store) != cudaSuccess) {
        cudaGetLastError();
        return dc_fail(ctx, DC_ERR_CUDA, "cudaIpcGetMemHandle of the store failed");
    }
    static_assert(sizeof(h) == DC_IPC_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle_out, &h, sizeof(h));
    return DC_OK;
}

int dc_store_attach_source(dc_ctx* ctx, const void* handle) {
    if (!ctx || !handle) return DC_ERR_INVALID_ARG;
    if (ctx->src_store) return dc_fail(ctx, DC_ERR_INVALID_ARG, "a source store is attached");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return dc_fail(ctx, DC_ERR_CUDA, "cudaIpcOpenMemHandle of the source store failed");
    }
    ctx->src_store = p;
    return DC_OK;
}

int dc_store_pull_slots(dc_ctx* ctx, int first, int count, dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    if (!ctx->src_store) return dc_fail(ctx, DC_ERR_NOT_READY, "no source store attached");
    if (first < 0 || count < 0 || first + count > ctx->cfg.max_frames)
        return dc_fail(ctx, DC_ERR_INVALID_ARG, "slot range outside [0, max_frames)");
    if (count == 0) return DC_OK;
    const long long slot_bytes = ctx->frame_rows * ctx->cfg.channels * ctx->elem_bytes;
    if (cudaMemcpyAsync(static_cast<char*>(ctx->store) + first * slot_bytes,
                        static_cast<const char*>(ctx->src_store) + first * slot_bytes,
                        (size_t)(count * slot_bytes), cudaMemcpyDeviceToDevice,
                        (cudaStream_t)stream) != cudaSuccess) {
        cudaGetLastError();
        return dc_fail(ctx, DC_ERR_CUDA, "copying slots from the source store failed");
    }
    return DC_OK;
}

int dc_sync_signal(dc_ctx* ctx, int word, unsigned value, int remote, dc_stream_t stream) {
    if (!ctx || word < 0 || word >= kSyncWords) return DC_ERR_INVALID_ARG;
    if (remote && !ctx->src_store) return dc_fail(ctx, DC_ERR_NOT_READY, "no source store attached");
    static StreamValueFn fn = stream_value_fn("cuStreamWriteValue32");
    if (!fn) return dc_fail(ctx, DC_ERR_UNSUPPORTED, "cuStreamWriteValue32 unavailable");
    if (fn((CUstream)stream, sync_word(ctx, word, remote != 0), value, 0) != CUDA_SUCCESS)
        return dc_fail(ctx, DC_ERR_CUDA, "cuStreamWriteValue32 failed");
    return DC_OK;
}

int dc_sync_wait(dc_ctx* ctx, int word, unsigned value, int remote, dc_stream_t stream) {
    if (!ctx || word < 0 || word >= kSyncWords) return DC_ERR_INVALID_ARG;
    if (remote && !ctx->src_store) return dc_fail(ctx, DC_ERR_NOT_READY, "no source store attached");
    static StreamValueFn fn = stream_value_fn("cuStreamWaitValue32");
    if (!fn) return dc_fail(ctx, DC_ERR_UNSUPPORTED, "cuStreamWaitValue32 unavailable");
    // CU_STREAM_WAIT_VALUE_GEQ: counters only grow
    if (fn((CUstream)stream, sync_word(ctx, word, remote != 0), value, 0x0) != CUDA_SUCCESS)
        return dc_fail(ctx, DC_ERR_CUDA, "cuStreamWaitValue32 failed");
    return DC_OK;
}

int dc_build_volume(dc_ctx* ctx, const int* ii, const int* jj, int M, float* const* vols,
                    dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    int rc = validate_edges(ctx, ii, jj, M);
    if (rc) return rc;
    if (!vols || !vols[0]) return dc_fail(ctx, DC_ERR_INVALID_ARG, "vols[0] is NULL");
    if (ctx->cfg.precision == DC_PREC_FP32X3)
        return dc_fail(ctx, DC_ERR_UNSUPPORTED, "DC_PREC_FP32X3 serves the fused lookup only");
    if (M == 0) return DC_OK;
    rc = ctx->tc_ready ? dc_launch_volume_tc(ctx, ii, jj, M, vols[0], (cudaStream_t)stream)
                       : dc_launch_volume_ffma(ctx, ii, jj, M, vols[0], (cudaStream_t)stream);
    if (rc) return rc;
    return dc_launch_volume_pyramid(ctx, vols, M, (cudaStream_t)stream);
}

int dc_pool_2x2(const float* in, float* out, long long N, int H, int W, dc_stream_t stream) {
    if (N < 0 || H < 0 || W < 0) return DC_ERR_INVALID_ARG;
    if (N == 0 || H < 2 || W < 2) return DC_OK;
    if (!in || !out) return DC_ERR_INVALID_ARG;
    return dc_launch_pool2x2(in, out, N, H, W, (cudaStream_t)stream);
}

int dc_lookup(dc_ctx* ctx, const float* const* vols, const float* coords, float* out, int M,
              dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    if (M < 0) return dc_fail(ctx, DC_ERR_INVALID_ARG, "M < 0");
    if (M == 0) return DC_OK;
    if (!vols || !coords || !out) return dc_fail(ctx, DC_ERR_INVALID_ARG, "NULL pointer");
    for (int l = 0; l < ctx->cfg.levels; l++)
        if (!vols[l]) return dc_fail(ctx, DC_ERR_INVALID_ARG, "vols[l] is NULL");
    return dc_launch_lookup(ctx, vols, coords, out, M, false, (cudaStream_t)stream);
}

int dc_lookup_single(dc_ctx* ctx, const float* const* vols, const float* coords, float* out,
                     dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    if (!vols || !coords || !out) return dc_fail(ctx, DC_ERR_INVALID_ARG, "NULL pointer");
    for (int l = 0; l < ctx->cfg.levels; l++)
        if (!vols[l]) return dc_fail(ctx, DC_ERR_INVALID_ARG, "vols[l] is NULL");
    return dc_launch_lookup(ctx, vols, coords, out, 1, true, (cudaStream_t)stream);
}

int dc_build_and_lookup(dc_ctx* ctx, const int* ii, const int* jj, int M, const float* coords,
                        float* out, dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    int rc = validate_edges(ctx, ii, jj, M);
    if (rc) return rc;
    if (M == 0) return DC_OK;
    if (!coords || !out) return dc_fail(ctx, DC_ERR_INVALID_ARG, "NULL pointer");
    if (ctx->tc_ready) return dc_launch_tc(ctx, ii, jj, M, coords, out, (cudaStream_t)stream);
    return dc_launch_alt(ctx, ii, jj, M, coords, out, (cudaStream_t)stream);
}

int dc_alt_lookup(dc_ctx* ctx, const int* ii, const int* jj, int M, const float* coords,
                  float* out, dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    int rc = validate_edges(ctx, ii, jj, M);
    if (rc) return rc;
    if (M == 0) return DC_OK;
    if (!coords || !out) return dc_fail(ctx, DC_ERR_INVALID_ARG, "NULL pointer");
    if (ctx->cfg.precision == DC_PREC_FP32X3)
        return dc_fail(ctx, DC_ERR_UNSUPPORTED, "DC_PREC_FP32X3 serves the fused lookup only");
    return dc_launch_alt(ctx, ii, jj, M, coords, out, (cudaStream_t)stream);
}

int dc_project(dc_ctx* ctx, const float* poses, const float* disps, const float* intrinsics,
               int num_frames, const int* ii, const int* jj, int M, float* coords, float* valid,
               dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    int rc = validate_edges(ctx, ii, jj, M);
    if (rc) return rc;
    if (num_frames < 1) return dc_fail(ctx, DC_ERR_INVALID_ARG, "num_frames < 1");
    if (M == 0) return DC_OK;
    if (!poses || !disps || !intrinsics || !coords)
        return dc_fail(ctx, DC_ERR_INVALID_ARG, "NULL pointer");
    return dc_launch_project(ctx, poses, disps, intrinsics, ii, jj, M, num_frames, coords, valid,
                             (cudaStream_t)stream);
}

int dc_project_build_and_lookup(dc_ctx* ctx, const float* poses, const float* disps,
                                const float* intrinsics, int num_frames, const int* ii,
                                const int* jj, int M, float* coords, float* valid, float* out,
                                dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    if (M > 0 && !out) return dc_fail(ctx, DC_ERR_INVALID_ARG, "NULL pointer");
    int rc = dc_project(ctx, poses, disps, intrinsics, num_frames, ii, jj, M, coords, valid,
                        stream);
    if (rc) return rc;
    return dc_build_and_lookup(ctx, ii, jj, M, coords, out, stream);
}

int dc_scatter_mean(dc_ctx* ctx, const float* feats, long long F, const int* ii_host, int E,
                    float* agg, int* kf_ids_host, int* K_out, dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    if (K_out) *K_out = 0;
    if (E < 0 || E > ctx->cfg.max_edges)
        return dc_fail(ctx, DC_ERR_INVALID_ARG,
                       "E=" + std::to_string(E) + " outside [0, max_edges=" +
                           std::to_string(ctx->cfg.max_edges) + "]");
    if (F < 1) return dc_fail(ctx, DC_ERR_INVALID_ARG, "F < 1");
    if (E == 0) return DC_OK;
    if (!feats || !ii_host || !agg) return dc_fail(ctx, DC_ERR_INVALID_ARG, "NULL pointer");
    return dc_scatter_mean_impl(ctx, feats, F, ii_host, E, agg, kf_ids_host, K_out,
                                (cudaStream_t)stream);
}

int dc_gather_rows(dc_ctx* ctx, const float* src, long long F, int num_rows, const int* idx,
                   int n, float* dst, dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    if (n < 0 || n > 65535) return dc_fail(ctx, DC_ERR_INVALID_ARG, "n outside [0, 65535]");
    if (F < 1 || num_rows < 1) return dc_fail(ctx, DC_ERR_INVALID_ARG, "F < 1 or num_rows < 1");
    if (n == 0) return DC_OK;
    if (!src || !idx || !dst) return dc_fail(ctx, DC_ERR_INVALID_ARG, "NULL pointer");
    return dc_gather_rows_impl(ctx, src, F, num_rows, idx, n, dst, (cudaStream_t)stream);
}

int dc_set_corr_encoder(dc_ctx* ctx, const float* weight, const float* bias, int out_channels,
                        dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    if (!weight || !bias) return dc_fail(ctx, DC_ERR_INVALID_ARG, "NULL pointer");
    return dc_set_corr_encoder_impl(ctx, weight, bias, out_channels, (cudaStream_t)stream);
}

int dc_corr_encode(dc_ctx* ctx, const float* corr, int M, void* out, dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    if (M < 0) return dc_fail(ctx, DC_ERR_INVALID_ARG, "M < 0");
    if (M == 0) return DC_OK;
    if (!corr || !out) return dc_fail(ctx, DC_ERR_INVALID_ARG, "NULL pointer");
    return dc_launch_encoder(ctx, corr, M, out, (cudaStream_t)stream);
}

int dc_build_lookup_encode(dc_ctx* ctx, const int* ii, const int* jj, int M, const float* coords,
                           float* corr, void* out, dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    if (!ctx->enc_ready)
        return dc_fail(ctx, DC_ERR_NOT_READY, "dc_set_corr_encoder has not been called");
    if (M > 0 && (!corr || !out)) return dc_fail(ctx, DC_ERR_INVALID_ARG, "NULL pointer");
    int rc = dc_build_and_lookup(ctx, ii, jj, M, coords, corr, stream);
    if (rc) return rc;
    return dc_corr_encode(ctx, corr, M, out, stream);
}

int dc_device_status(dc_ctx* ctx, dc_stream_t stream) {
    if (!ctx) return DC_ERR_INVALID_ARG;
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess)
        return dc_fail(ctx, DC_ERR_CUDA, cudaGetErrorString(cudaGetLastError()));
    int v = 0;
    if (cudaMemcpy(&v, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
        return dc_fail(ctx, DC_ERR_CUDA, "reading the device error word failed");
    if (v != 0) {
        cudaMemset(ctx->dev_err, 0, sizeof(int));
        return dc_fail(ctx, DC_ERR_DEVICE_TIMEOUT,
                       "a device-side wait timed out (site " + std::to_string(v) + ")");
    }
    return DC_OK;
}

}  // extern "C"

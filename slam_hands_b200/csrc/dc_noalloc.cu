// dc_noalloc.cu -- dc_build_and_lookup_static: the fused build + pyramid +
// lookup for callers that cannot allocate device memory.
//
// Some hosts of this library may not call cudaMalloc at all: a process whose
// device memory is owned by another allocator (a caching pool that must see
// every allocation, a fixed pre-partitioned arena on a shared GPU), or code that
// runs where allocating would synchronise the device or fail for lack of
// memory at an unpredictable moment.  For them this entry point takes no
// context: the packed keyframe store that dc_build_and_lookup keeps in its
// context lives here in one file-scope device array of fixed size, shared by
// all calls in the process on a given GPU.
#include <cstdio>
#include <mutex>

#include "dc_internal.cuh"

namespace {

// 32 MiB: room for 18 keyframes of a 54x96x128 fp16 pyramid (1.84 MB each),
// or 31 of 48x64x128 (1.08 MB each).  Every GPU that loads the library holds it
// until exit.
constexpr size_t kScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];
static __device__ int g_scratch_err;

// Device addresses of the arrays, looked up once per device (host code may not
// use the symbols themselves: on the host they are stand-ins, not addresses).
struct DeviceScratch {
    bool ready = false;
    void* store = nullptr;
    int* err = nullptr;
};
DeviceScratch g_dev[kMaxDevices];
std::mutex g_dev_mutex;  // first calls from several host threads fill g_dev safely

int scratch_for_device(int dev, DeviceScratch** out) {
    if (dev < 0 || dev >= kMaxDevices) return DC_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    DeviceScratch& d = g_dev[dev];
    if (!d.ready) {
        void* store = nullptr;
        int* err = nullptr;
        if (cudaGetSymbolAddress(&store, g_scratch) != cudaSuccess ||
            cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_scratch_err) != cudaSuccess) {
            cudaGetLastError();
            return DC_ERR_CUDA;
        }
        d.store = store;
        d.err = err;
        d.ready = true;
    }
    *out = &d;
    return DC_OK;
}

// Diagnostics go to stderr: this entry point has no context to keep a message.
int fail(int status, const char* msg) {
    std::fprintf(stderr, "dc_build_and_lookup_static: %s\n", msg);
    return status;
}

}  // namespace

extern "C" {

int dc_build_and_lookup_static(const dc_config* cfg, const void* fmaps, int dtype,
                               int num_frames, const int* ii, const int* jj, int M,
                               const float* coords, float* out, dc_stream_t stream) {
    if (!cfg) return fail(DC_ERR_INVALID_ARG, "cfg is NULL");
    const dc_config& c = *cfg;
    if (dtype != DC_DTYPE_F32 && dtype != DC_DTYPE_F16)
        return fail(DC_ERR_INVALID_ARG, "dtype must be DC_DTYPE_F32 or DC_DTYPE_F16");
    if (num_frames < 1 || M < 0) return fail(DC_ERR_INVALID_ARG, "num_frames < 1 or M < 0");
    if (M == 0) return DC_OK;
    if (!fmaps || !ii || !jj || !coords || !out) return fail(DC_ERR_INVALID_ARG, "NULL pointer");

    // the context a dc_create would build, on the stack, over the static store
    dc_ctx ctx;
    if (dc_init_geometry(&ctx, c, num_frames) != DC_OK)
        return fail(DC_ERR_INVALID_ARG, "invalid dc_config");
    ctx.cfg.max_frames = num_frames;
    ctx.cfg.max_edges = M;
    if (ctx.store_bytes > (long long)kScratchBytes) {
        char msg[200];
        std::snprintf(msg, sizeof msg,
                      "%d frames need %lld bytes of packed store; the static scratch holds %lld",
                      num_frames, ctx.store_bytes, (long long)kScratchBytes);
        return fail(DC_ERR_INVALID_ARG, msg);
    }
    if (cudaGetDevice(&ctx.device) != cudaSuccess) return fail(DC_ERR_CUDA, "cudaGetDevice failed");
    cudaDeviceGetAttribute(&ctx.num_sms, cudaDevAttrMultiProcessorCount, ctx.device);
    DeviceScratch* ds = nullptr;
    int rc = scratch_for_device(ctx.device, &ds);
    if (rc) return fail(rc, "cudaGetSymbolAddress of the static scratch failed");
    ctx.store = ds->store;
    ctx.dev_err = ds->err;

    cudaStream_t s = (cudaStream_t)stream;
    // The previous call left its contents behind.  The packing kernel rewrites
    // every data row; the padding rows (read as zero operand rows by the
    // tensor-core kernel) are cleared here.  The error word is not cleared: it
    // keeps a time-out until dc_static_device_status reads it.
    rc = dc_launch_store_zero_padding(&ctx, 0, num_frames, s);
    if (rc) return fail(rc, ctx.err.c_str());
    rc = dc_launch_store(&ctx, fmaps, dtype, 0, num_frames, s);
    if (rc) return fail(rc, ctx.err.c_str());
    if (dc_tc_supported(&ctx)) {
        rc = dc_tc_prepare(&ctx);
        if (rc) return fail(rc, ctx.err.c_str());
        rc = dc_launch_tc(&ctx, ii, jj, M, coords, out, s);
    } else {
        rc = dc_launch_alt(&ctx, ii, jj, M, coords, out, s);
    }
    if (rc) return fail(rc, ctx.err.c_str());
    return DC_OK;
}

int dc_static_device_status(dc_stream_t stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(DC_ERR_CUDA, "cudaGetDevice failed");
    DeviceScratch* ds = nullptr;
    if (scratch_for_device(dev, &ds) != DC_OK)
        return fail(DC_ERR_CUDA, "cudaGetSymbolAddress of the static error word failed");
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) {
        cudaGetLastError();
        return fail(DC_ERR_CUDA, "synchronising the stream failed");
    }
    int v = 0;
    if (cudaMemcpy(&v, ds->err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
        return fail(DC_ERR_CUDA, "reading the static error word failed");
    if (v == 0) return DC_OK;
    if (cudaMemset(ds->err, 0, sizeof(int)) != cudaSuccess)
        return fail(DC_ERR_CUDA, "clearing the static error word failed");
    char msg[96];
    std::snprintf(msg, sizeof msg, "a device-side wait timed out (site %d)", v);
    return fail(DC_ERR_DEVICE_TIMEOUT, msg);
}

}  // extern "C"

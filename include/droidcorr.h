/*
 * droidcorr.h -- C ABI of the B200 (sm_100a) DROID-SLAM correlation library
 * (libdroidcorr.so).
 *
 * It replaces the correlation hot path of slam-hands (cuda_slam/main.cu and its
 * copy in cuda_pipeline/slam.cuh):
 *
 *   reference                                             replaced by
 *   ----------------------------------------------------  ---------------------------
 *   DroidState::fmaps / add_keyframe  main.cu:677, :755    dc_set_frames
 *   CudaDroid::build_correlation      main.cu:1500-1526    dc_build_volume (M = 1)
 *   (cublasGemmEx + cuDNN avg_pool2d, nn.cuh:389-410)
 *   avg_pool_2x2_kernel               main.cu:1150-1170    dc_pool_2x2
 *   CudaDroid::sample_correlation     main.cu:1529-1552    dc_lookup (M = 1)
 *   (corr_index_kernel                main.cu:1079-1114)
 *   batch_corr_sample_kernel x4       main.cu:1175-1217    dc_lookup
 *   CudaDroid::batch_build_and_sample_correlation          dc_build_and_lookup
 *                                     main.cu:1555-1613
 *   (no reference counterpart: on-the-fly lookup)          dc_alt_lookup
 *   projmap_kernel                    se3.cuh:118-177      dc_project
 *   + batch_coords_hw2_to_2hw         main.cu:1135-1146
 *   projmap + hw2_to_2hw + batch_build_and_sample_...      dc_project_build_and_lookup
 *                                     main.cu:2188-2201
 *   GraphAgg scatter_mean loop        main.cu:2255-2294    dc_scatter_mean
 *   per-edge inps[ii[e]] copy loop    main.cu:2215-2224    dc_gather_rows
 *   corr_enc_0 + relu + round_to_fp16 main.cu:552-553,      dc_set_corr_encoder,
 *   (UpdateModule::forward)           :603-606              dc_corr_encode,
 *                                                           dc_build_lookup_encode
 *   cuda_pipeline/slam.cuh:2796, :2825, :2851              the same three entry points
 *
 * Conventions (all entry points):
 *   - Every pointer argument named *_dev is DEVICE memory owned by the caller
 *     (the reference's GpuBuf buffers, nn.cuh:45-71).  The library owns only its
 *     context: the packed feature-map store and its scratch.
 *   - Work is enqueued on the given stream; no call synchronises the host except
 *     dc_create / dc_destroy.  A context may be used by one host thread at a time.
 *   - Return value: DC_OK (0) or a DC_ERR_* status.  Nothing exits the process
 *     (the reference's CUDA_CHECK -> exit(1), nn.cuh:17-41, is replaced by status
 *     codes).  dc_last_error() returns a message for the last failure.
 *
 * Layouts (identical to the reference):
 *   fmaps     [count][C][h][w]            fp32 or fp16, one slot per keyframe
 *   ii, jj    [M] int32 (device)           edge e correlates source frame ii[e]
 *                                          (pixels p) with target frame jj[e] (q)
 *   vol_l     [M][h*w][h>>l][w>>l] fp32    level-l volume, V_l[e][p][y][x]
 *   coords    [M][2][h][w] fp32            ch0 = x, ch1 = y, target pixels at 1/8 res
 *   out       [M][levels*(2r+1)^2][h][w]   channel l*(2r+1)^2 + a*(2r+1) + b,
 *                                          a = x offset, b = y offset (main.cu:1203-1213)
 */
#ifndef DROIDCORR_H_
#define DROIDCORR_H_

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t / CUstream. */
typedef struct CUstream_st* dc_stream_t;
typedef struct dc_ctx dc_ctx;

/* status codes */
#define DC_OK 0
#define DC_ERR_INVALID_ARG 1
#define DC_ERR_CUDA 2
#define DC_ERR_UNSUPPORTED 3
#define DC_ERR_NO_MEMORY 4
#define DC_ERR_DEVICE_TIMEOUT 5
#define DC_ERR_NOT_READY 6

/* Arithmetic of the correlation dot products (the volume build).
 *   DC_PREC_FP32    exact fp32 FFMA, channels accumulated in order c = 0..C-1
 *                   (CUDA cores; bit-exact materialised volume)
 *   DC_PREC_TF32    inputs rounded to TF32 (10 explicit mantissa bits, round to
 *                   nearest, ties away), fp32 accumulate on the tensor cores: a
 *                   TF32 value within fp16's normal range (2^-14 <= |x| < 65504)
 *                   is an fp16 value, so the store holds fp16 and the fp16
 *                   kernels run; smaller magnitudes keep fp16's (subnormal)
 *                   precision
 *   DC_PREC_BF16    inputs rounded to BF16, fp32 accumulate (tensor cores)
 *   DC_PREC_FP16    inputs rounded to FP16, fp32 accumulate (tensor cores) --
 *                   the reference's own arithmetic (FP16 fmaps, cublasGemmBatchedEx
 *                   with CUBLAS_COMPUTE_32F, main.cu:1573-1581)
 *   DC_PREC_FP32X3  fp32 accuracy on the tensor cores: every input is split into
 *                   hi = fp16(x) and lo = fp16(x - hi), and each dot product is
 *                   hi.hi + hi.lo + lo.hi (three fp16 passes, fp32 accumulation;
 *                   the dropped lo.lo term is ~2^-22 relative) -- within 1e-5 of
 *                   the fp32 result for inputs within fp16's range.  Serves
 *                   dc_build_and_lookup (and dc_project_build_and_lookup) only;
 *                   channels 64 or 128. */
#define DC_PREC_FP32 0
#define DC_PREC_TF32 1
#define DC_PREC_BF16 2
#define DC_PREC_FP16 3
#define DC_PREC_FP32X3 4

/* element type of caller feature maps */
#define DC_DTYPE_F32 0
#define DC_DTYPE_F16 1

typedef struct dc_config {
    int h, w;        /* feature grid (image / 8), e.g. 48 x 64 */
    int channels;    /* C: 32, 64, 128 or 256 (128 in DROID-SLAM) */
    int levels;      /* pyramid levels, 1..4 (reference: 4, main.cu:1604) */
    int radius;      /* lookup radius, 0..3 (reference: 3, main.cu:1531) */
    int max_frames;  /* keyframe slots in the store (DroidState::MAX_KEYFRAMES) */
    int max_edges;   /* largest M of one call (reference chunk: MAX_BATCH_EDGES = 48) */
    int precision;   /* DC_PREC_* */
    float alpha;     /* volume scale; the reference uses 1/16 (main.cu:1506, :1572) */
} dc_config;

/* Fill *cfg with the reference defaults for an h x w grid:
 * C = 128, levels = 4, radius = 3, max_frames = 512, max_edges = 48,
 * precision = DC_PREC_FP16, alpha = 1/16. */
void dc_default_config(dc_config* cfg, int h, int w);

/* Create a context on the current CUDA device.  Allocates the feature-map store
 * (max_frames slots).  Replaces the correlation part of CudaDroid::init,
 * main.cu:1405-1426. */
int dc_create(const dc_config* cfg, dc_ctx** out);
int dc_destroy(dc_ctx* ctx);
const char* dc_last_error(const dc_ctx* ctx);
const char* dc_status_string(int status);

/* Bytes of device memory the context holds: the packed store and its sync
 * page, the error word and lists, and what later calls allocated (encoder
 * weights, tile-order scratch). */
long long dc_context_bytes(const dc_ctx* ctx);

/* Pack `count` feature maps into store slots first_slot .. first_slot+count-1
 * (the library's resident copy of DroidState::fmaps, main.cu:677, written by
 * add_keyframe, main.cu:755).  fmaps_dev: [count][C][h][w], dtype DC_DTYPE_*.
 * The store keeps, per slot, the map and its 2x2-average pyramid in the
 * precision's element type, pixel-major.  Must be called again for a slot
 * whenever its feature map changes. */
int dc_set_frames(dc_ctx* ctx, const void* fmaps_dev, int dtype, int first_slot, int count,
                  dc_stream_t stream);

/* Device address and byte size of store slots first_slot .. first_slot+count-1
 * (contiguous).  For replicating packed keyframes to other GPUs (e.g. one NCCL
 * broadcast of the packed slots instead of re-packing on every GPU).  No
 * reference counterpart: the reference runs on one GPU. */
int dc_store_slots(dc_ctx* ctx, int first_slot, int count, void** ptr_out,
                   long long* bytes_out);

/* Replication of packed keyframes between processes (one per GPU) through the
 * copy engines over NVLink, no SMs involved: the owner exports its store with
 * dc_store_ipc_handle (DC_IPC_HANDLE_BYTES bytes, a CUDA IPC memory handle, to
 * be passed to the other processes by the host); each other process attaches
 * it once with dc_store_attach_source -- both contexts must have been created
 * with the same dc_config -- and copies slots with dc_store_pull_slots, an
 * asynchronous device-to-device copy on `stream`.  The caller orders the pull
 * after the owner's dc_set_frames of those slots (e.g. an interprocess CUDA
 * event) and keeps the owner from rewriting slots being pulled.  No reference
 * counterpart: the reference runs on one GPU. */
#define DC_IPC_HANDLE_BYTES 64
int dc_store_ipc_handle(dc_ctx* ctx, void* handle_out);
int dc_store_attach_source(dc_ctx* ctx, const void* handle);
int dc_store_pull_slots(dc_ctx* ctx, int first_slot, int count, dc_stream_t stream);

/* Stream-ordered counters for that replication, with no host round trip and
 * no SM: every store carries a page of 1024 32-bit words (zero at creation).
 * dc_sync_signal writes `value` to word `word` of this context's page
 * (remote = 0) or of the attached source's page over NVLink (remote = 1) once
 * the stream's earlier work is done; dc_sync_wait holds the stream until that
 * word is >= value (cuStreamWriteValue32 / cuStreamWaitValue32).  Counters are
 * meant to grow (e.g. the step index + 1).  A wait whose value never comes
 * holds its stream until the process ends: use them between processes that
 * run the same step sequence, with host-side liveness checks between steps. */
int dc_sync_signal(dc_ctx* ctx, int word, unsigned value, int remote, dc_stream_t stream);
int dc_sync_wait(dc_ctx* ctx, int word, unsigned value, int remote, dc_stream_t stream);

/* Materialised volumes for M edges (CudaDroid::build_correlation, main.cu:1500,
 * and steps 1-3 of batch_build_and_sample_correlation, main.cu:1558-1596):
 * vol0 = alpha * f_ii^T f_jj, then vol_l = 2x2 average of vol_{l-1} over the
 * target axes (cascaded, floor on odd dims).  vols_dev: host array of `levels`
 * device pointers; entries 1.. may be NULL to skip those levels. */
int dc_build_volume(dc_ctx* ctx, const int* ii_dev, const int* jj_dev, int M,
                    float* const* vols_dev, dc_stream_t stream);

/* One 2x2 average-pool level, in [N][H][W] -> out [N][H/2][W/2]
 * (avg_pool_2x2_kernel, main.cu:1150-1170).  Bit-identical to the reference. */
int dc_pool_2x2(const float* in_dev, float* out_dev, long long N, int H, int W,
                dc_stream_t stream);

/* Radius-r bilinear lookup from materialised volumes (batch_corr_sample_kernel,
 * main.cu:1175-1217, all levels in one launch; out is written, not accumulated,
 * so no memset is needed).  vols_dev: host array of `levels` device pointers.
 * Bit-identical to the reference kernel for the same volumes. */
int dc_lookup(dc_ctx* ctx, const float* const* vols_dev, const float* coords_dev,
              float* out_dev, int M, dc_stream_t stream);

/* The corr_index_kernel arithmetic (single-edge sample_correlation,
 * main.cu:1529-1552: each tap's weighted value rounded, then added). */
int dc_lookup_single(dc_ctx* ctx, const float* const* vols_dev, const float* coords_dev,
                     float* out_dev, dc_stream_t stream);

/* Build + pyramid + lookup for M edges without storing any volume
 * (batch_build_and_sample_correlation, main.cu:1555-1613).  Reads source and
 * target maps from store slots ii[e], jj[e].  Pooled levels are computed as
 * alpha * <f_ii, P_l f_jj> (P_l = l-fold 2x2 average of the target map), equal to
 * pooling the volume because pooling is linear. */
int dc_build_and_lookup(dc_ctx* ctx, const int* ii_dev, const int* jj_dev, int M,
                        const float* coords_dev, float* out_dev, dc_stream_t stream);

/* On-the-fly ("alt-corr") lookup: same result as dc_build_and_lookup, computed as
 * per-pixel gathered dot products against the pooled target maps (only the
 * (2r+2)^2 taps of each level), never forming a volume row.  Memory per edge is
 * the output only.  No reference counterpart (the reference always
 * materialises, main.cu:2185-2201). */
int dc_alt_lookup(dc_ctx* ctx, const int* ii_dev, const int* jj_dev, int M,
                  const float* coords_dev, float* out_dev, dc_stream_t stream);

/* Reprojection of every source pixel of edge e into frame jj[e]
 * (projmap_kernel, se3.cuh:118-177, followed by the layout pass
 * batch_coords_hw2_to_2hw, main.cu:1135-1146, as one kernel):
 *   poses_dev      [num_frames][7]   t_x t_y t_z q_x q_y q_z q_w (world -> camera)
 *   disps_dev      [num_frames][h][w] inverse depth
 *   intrinsics_dev [4]               fx fy cx cy (at the feature-map resolution)
 *   coords_dev     [M][2][h][w]      written: x then y, the layout dc_lookup and
 *                                    dc_build_and_lookup read
 *   valid_dev      [M][h][w] or NULL written: 1 where the projected depth
 *                                    exceeds 0.25 (MIN_DEPTH), else 0
 * Pixels whose projected depth is at most 0.01, and all pixels of an edge whose
 * ii/jj lies outside [0, num_frames), keep their own coordinates (u, v).
 * Coordinates agree with the reference kernel to a few float ulps: the
 * reference is built with --use_fast_math (approximate division). */
int dc_project(dc_ctx* ctx, const float* poses_dev, const float* disps_dev,
               const float* intrinsics_dev, int num_frames, const int* ii_dev,
               const int* jj_dev, int M, float* coords_dev, float* valid_dev,
               dc_stream_t stream);

/* dc_project followed by dc_build_and_lookup on the projected coordinates: the
 * reference's per-batch steps 1-3 (main.cu:2188-2201: projmap_kernel, the
 * layout pass and batch_build_and_sample_correlation) in two kernels, with no
 * interleaved coordinate buffer.  coords_dev [M][2][h][w] receives the
 * coordinates (the motion features downstream need them, main.cu:2206-2211);
 * valid_dev may be NULL. */
int dc_project_build_and_lookup(dc_ctx* ctx, const float* poses_dev, const float* disps_dev,
                                const float* intrinsics_dev, int num_frames,
                                const int* ii_dev, const int* jj_dev, int M,
                                float* coords_dev, float* valid_dev, float* out_dev,
                                dc_stream_t stream);

/* GraphAgg scatter-mean (main.cu:2255-2294): for every keyframe k that is the
 * source of some edge, agg[k'] = mean over edges e with ii[e] == k of feats[e],
 * k' = k's rank among those keyframes in ascending id order (the reference's
 * std::set).  One kernel replaces the reference's memset + one scale_add_kernel
 * launch per edge + one per keyframe, and reproduces its floats bit for bit: a
 * running fp32 sum from 0 in edge order, then x + (1/n - 1) x as one fused
 * multiply-add for keyframes with n > 1 edges.
 *   feats_dev    [E][F]   per-edge features (F = 128*h*w in the reference)
 *   ii_host      [E]      HOST array of source keyframes (state.ii_host)
 *   agg_dev      [K][F]   written, K = number of distinct ii (<= E)
 *   kf_ids_host  [>= K] or NULL: receives the keyframe id of each agg row
 *   K_out        or NULL: receives K
 * E <= max_edges.  The edge lists are copied from the host on `stream`
 * (pageable memory: the call returns once the host data is staged) into a
 * small buffer of the context, so two dc_scatter_mean calls on one context
 * must not overlap on the GPU (use one stream per context, or separate
 * contexts). */
int dc_scatter_mean(dc_ctx* ctx, const float* feats_dev, long long F, const int* ii_host, int E,
                    float* agg_dev, int* kf_ids_host, int* K_out, dc_stream_t stream);

/* Row gather for the update step's per-edge loads (main.cu:2215-2224, one
 * synchronous cudaMemcpy per edge: batch_inps[e] = inps[ii[bs + e]]):
 * dst_dev[e] = src_dev[idx_dev[e]] for e < n, rows of F floats, one launch on
 * `stream`.  src_dev [num_rows][F], idx_dev [n] (device), dst_dev [n][F].
 * Rows whose index is outside [0, num_rows) are written as zeros.  n <= 65535.
 * (The loop's contiguous copies, edge_nets <-> batch_nets and batch_agg1 ->
 * all_agg1, are single ranges: one cudaMemcpyAsync each.) */
int dc_gather_rows(dc_ctx* ctx, const float* src_dev, long long F, int num_rows,
                   const int* idx_dev, int n, float* dst_dev, dc_stream_t stream);

/* The update operator's correlation encoder, first layer (UpdateModule
 * corr_enc_0: a 1x1 convolution levels*(2r+1)^2 = 196 -> 128 with bias,
 * main.cu:552-553, then relu_inplace and round_to_fp16, main.cu:603-606), on
 * the tensor cores.  dc_set_corr_encoder packs the layer's weights once:
 *   weight_dev [128][196] fp32 (the convolution's [co][ci][1][1] weights)
 *   bias_dev   [128] fp32;  out_channels must be 128.
 * The context allocates 64 KB for the packed weights on the first call. */
int dc_set_corr_encoder(dc_ctx* ctx, const float* weight_dev, const float* bias_dev,
                        int out_channels, dc_stream_t stream);

/* out = fp16(relu(W corr + b)) per pixel: corr_dev [M][196][h][w] fp32 (the
 * lookup's output), out_dev [M][128][h][w] fp16 -- the values the reference
 * holds as fp16-rounded floats, stored in half the bytes.  Features and
 * weights are rounded to fp16 for the tensor cores, fp32 accumulation. */
int dc_corr_encode(dc_ctx* ctx, const float* corr_dev, int M, void* out_dev, dc_stream_t stream);

/* dc_build_and_lookup into corr_dev (caller-owned [M][196][h][w], the
 * reference's batch_corr buffer, main.cu:1336), then dc_corr_encode into
 * out_dev: the update step's correlation features and their encoding
 * (main.cu:2200 then :603-606) back to back, so that the 196-channel features
 * are read by the encoder while they are still in L2. */
int dc_build_lookup_encode(dc_ctx* ctx, const int* ii_dev, const int* jj_dev, int M,
                           const float* coords_dev, float* corr_dev, void* out_dev,
                           dc_stream_t stream);

/* Wait for `stream`, then report and clear the device error word that the
 * library's bounded device-side waits raise when they time out: DC_OK or
 * DC_ERR_DEVICE_TIMEOUT.  (The reference has no device-side waits.) */
int dc_device_status(dc_ctx* ctx, dc_stream_t stream);

/* dc_build_and_lookup for callers that may not allocate device memory (no
 * counterpart in the reference).  Some hosts cannot call cudaMalloc: their
 * device memory belongs to another allocator or a fixed arena, or allocating
 * would synchronise the GPU at a bad moment.  This call needs no context: it
 * packs `num_frames` feature maps (fmaps_dev [num_frames][C][h][w], dtype
 * DC_DTYPE_*) into a library-owned static device array of 32 MiB and runs the
 * fused build + pyramid + lookup for M edges into out_dev, allocating nothing.
 *   - cfg is read as for dc_create (max_frames / max_edges are ignored);
 *     a packed store larger than 32 MiB is rejected with DC_ERR_INVALID_ARG
 *     (fp16 at 48x64x128: 31 frames; at 54x96x128: 18 frames).
 *   - The array belongs to the current device and is kept until the process
 *     exits; the first call on each device looks up its address
 *     (cudaGetSymbolAddress), so make that first call before any stream
 *     capture.  Each call clears the parts that must start at zero (the
 *     padding rows of the packed store).
 *   - A bounded device-side wait that times out leaves `out` incomplete and is
 *     reported by dc_static_device_status, not by this call's return value
 *     (the call does not wait for the GPU).
 *   - All calls share the one array: calls that overlap on the GPU (other
 *     streams, other host threads) race and must be serialised by the caller.
 *   - Diagnostics go to stderr (there is no context for dc_last_error). */
int dc_build_and_lookup_static(const dc_config* cfg, const void* fmaps_dev, int dtype,
                               int num_frames, const int* ii_dev, const int* jj_dev, int M,
                               const float* coords_dev, float* out_dev, dc_stream_t stream);

/* Status of dc_build_and_lookup_static on the current device: waits for
 * `stream`, then reports and clears the device error word of the static store
 * (the counterpart of dc_device_status, which needs a context).  DC_OK, or
 * DC_ERR_DEVICE_TIMEOUT when a bounded device-side wait of an earlier static
 * call timed out -- that call's output is then incomplete.  The word keeps a
 * time-out until this call reads it; all static calls on the device share it.
 * Allocates nothing. */
int dc_static_device_status(dc_stream_t stream);

/* Test hook of the bounded device-side waits.  With wait_limit_ns > 0, every
 * later launch of the fused tensor-core kernel in this process (all contexts
 * and the static entry point) makes each CTA withhold its first source-tile
 * load, so that the MMA warp's wait for it -- limited to wait_limit_ns instead
 * of 2 s -- can end only by time-out.  The kernel then raises the device error
 * word (DC_ERR_DEVICE_TIMEOUT from dc_device_status / dc_static_device_status),
 * lets its copies in flight land, frees its tensor memory and returns; its
 * output is incomplete and the context stays usable.  0 restores normal
 * operation.  Change it only while no fused kernel is being launched from
 * another host thread.  No reference counterpart (the reference has no
 * device-side waits). */
int dc_debug_inject_stall(long long wait_limit_ns);

/* Cap the CTAs of the persistent fused tensor-core kernel (dc_build_and_lookup,
 * fp16 / bf16) at max_ctas; 0 (the default) runs one CTA per SM.  Each CTA
 * holds a whole SM, so a kernel on another stream -- e.g. the NCCL broadcast
 * of the next step's keyframe -- can only run beside it on SMs left free.
 * Results do not depend on the cap.  No reference counterpart (one GPU, one
 * stream in the reference). */
int dc_set_max_ctas(dc_ctx* ctx, int max_ctas);

/* Order in which the fused tensor-core kernel (dc_build_and_lookup and the
 * calls built on it, fp16 / bf16 / tf32 / fp32x3) groups an edge's source
 * pixels into its 128-pixel tiles.  A tile multiplies its pixels against every
 * target row that any of their windows touches, so the order sets how many
 * target rows each tile streams:
 *   DC_ORDER_SOURCE      128 consecutive source pixels (the default): compact
 *                        when the flow is smooth, nearly the whole level when
 *                        neighbouring pixels' windows scatter (large, noisy
 *                        flow -- the backend's N(0, 8 px) graphs);
 *   DC_ORDER_WINDOW_ROW  a pre-pass sorts each edge's pixels by the row of
 *                        their level-0 window (stable, ties by pixel index); a
 *                        tile's windows then share a few rows, at the price of
 *                        scattered output stores and a gathered source tile;
 *   DC_ORDER_AUTO        the pre-pass picks, per edge, the window-row order
 *                        when the level-0 target pixels it saves per tile
 *                        reach 8 x the output channels (1568 at r = 3, four
 *                        levels), else the source order.
 * Results do not depend on the order (each output is computed from its own
 * pixel's dot products).  The first call with an order other than
 * DC_ORDER_SOURCE allocates the permutation scratch (4 bytes per pixel and
 * edge, max_edges edges); grids taller than 496 rows keep the source order.
 * The pre-pass is one more launch per call, and calls on one context share
 * the scratch (one call in flight per context).  No reference counterpart: the reference's volume
 * build has no tiles (main.cu:1555-1613). */
#define DC_ORDER_SOURCE 0
#define DC_ORDER_WINDOW_ROW 1
#define DC_ORDER_AUTO 2
int dc_set_tile_order(dc_ctx* ctx, int order);

/* Number of kernel launches the library has issued on this context (for
 * launch accounting in benchmarks). */
long long dc_launch_count(const dc_ctx* ctx);

#ifdef __cplusplus
}
#endif
#endif /* DROIDCORR_H_ */

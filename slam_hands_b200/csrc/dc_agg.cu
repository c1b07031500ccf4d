// dc_agg.cu -- GraphAgg scatter-mean: the mean of the per-edge features over
// the edges that share a source keyframe, for every keyframe that has an edge.
//
// Replaces the reference's host loop (cuda_slam/main.cu:2255-2294): a memset of
// the compact per-keyframe buffer, one scale_add_kernel launch per edge
// (dst += 1 * src, nn.cuh:382-385) and one per keyframe with more than one edge
// (dst += (1/count - 1) * dst).  Here one kernel does it: CTA (k, chunk) owns
// keyframe k's slice of F features, adds its edges' slices in edge order and
// scales once, so every output float is the reference's: a running fp32 sum
// from +0 in the order of the edge list, then fmaf(1/count - 1, sum, sum) with
// 1/count - 1 formed on the host in fp32 (nvcc contracts `dst += s * src` to
// one fused multiply-add).  HBM-bound: E*F floats read once, K*F written once.
//
// The compact keyframe order is ascending keyframe id, as the reference's
// std::set; the per-keyframe edge lists are built on the host from ii (the
// reference's state.ii_host) and copied into the context's small device
// allocation.
#include <algorithm>
#include <cstring>
#include <vector>

#include "dc_internal.cuh"

namespace {

constexpr int kAggThreads = 256;

// lists: order[E] (edges grouped by keyframe, in edge order), offs[K + 1],
// scale[K] (as float bits; 0 for keyframes with one edge).
template <bool kVec>
__global__ void __launch_bounds__(kAggThreads) scatter_mean_kernel(
    const float* __restrict__ feats, long long F, const int* __restrict__ order,
    const int* __restrict__ offs, const float* __restrict__ scale, float* __restrict__ agg) {
    const int k = blockIdx.y;
    const int e0 = offs[k], e1 = offs[k + 1];
    const float sc = scale[k];
    if (kVec) {
        const long long i = (long long)blockIdx.x * kAggThreads + threadIdx.x;  // float4 index
        if (i >= F / 4) return;
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        auto add = [&](const float4& v) {
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        };
        auto load = [&](int t) {
            return __ldcs(reinterpret_cast<const float4*>(feats + (size_t)order[t] * F) + i);
        };
        int t = e0;
        for (; t + 4 <= e1; t += 4) {  // four loads in flight, added in edge order
            const float4 v0 = load(t), v1 = load(t + 1), v2 = load(t + 2), v3 = load(t + 3);
            add(v0);
            add(v1);
            add(v2);
            add(v3);
        }
        for (; t < e1; t++) add(load(t));
        if (e1 - e0 > 1) {
            acc.x = fmaf(sc, acc.x, acc.x);
            acc.y = fmaf(sc, acc.y, acc.y);
            acc.z = fmaf(sc, acc.z, acc.z);
            acc.w = fmaf(sc, acc.w, acc.w);
        }
        reinterpret_cast<float4*>(agg + (size_t)k * F)[i] = acc;
    } else {
        const long long i = (long long)blockIdx.x * kAggThreads + threadIdx.x;
        if (i >= F) return;
        float acc = 0.0f;
        for (int t = e0; t < e1; t++) acc = __fadd_rn(acc, __ldcs(feats + (size_t)order[t] * F + i));
        if (e1 - e0 > 1) acc = fmaf(sc, acc, acc);
        agg[(size_t)k * F + i] = acc;
    }
}

}  // namespace

int dc_scatter_mean_impl(dc_ctx* ctx, const float* feats, long long F, const int* ii_host,
                         int E, float* agg, int* kf_ids_host, int* K_out, cudaStream_t s) {
    // compact keyframe order (ascending id) and stable per-keyframe edge lists
    std::vector<int> ids(ii_host, ii_host + E);
    std::sort(ids.begin(), ids.end());
    ids.erase(std::unique(ids.begin(), ids.end()), ids.end());
    const int K = (int)ids.size();
    if (K > 65535)  // one grid row per keyframe
        return dc_fail(ctx, DC_ERR_INVALID_ARG,
                       "more than 65535 distinct source keyframes in one call");
    std::vector<int> offs(K + 1, 0), order(E);
    std::vector<int> compact(E);
    for (int e = 0; e < E; e++) {
        compact[e] = (int)(std::lower_bound(ids.begin(), ids.end(), ii_host[e]) - ids.begin());
        offs[compact[e] + 1]++;
    }
    for (int k = 0; k < K; k++) offs[k + 1] += offs[k];
    {
        std::vector<int> fill(offs.begin(), offs.end() - 1);
        for (int e = 0; e < E; e++) order[fill[compact[e]]++] = e;
    }
    std::vector<int> lists(E + (K + 1) + K);
    std::copy(order.begin(), order.end(), lists.begin());
    std::copy(offs.begin(), offs.end(), lists.begin() + E);
    for (int k = 0; k < K; k++) {
        const int n = offs[k + 1] - offs[k];
        const float sc = n > 1 ? 1.0f / (float)n - 1.0f : 0.0f;
        std::memcpy(&lists[E + K + 1 + k], &sc, sizeof(float));
    }
    int* dl = ctx->dev_err + 32;
    if (cudaMemcpyAsync(dl, lists.data(), lists.size() * sizeof(int), cudaMemcpyHostToDevice,
                        s) != cudaSuccess)
        return dc_fail(ctx, DC_ERR_CUDA, "copying the scatter-mean lists failed");
    const int* d_order = dl;
    const int* d_offs = dl + E;
    const float* d_scale = reinterpret_cast<const float*>(dl + E + K + 1);
    const bool vec = (F % 4) == 0 && (reinterpret_cast<uintptr_t>(feats) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(agg) & 15) == 0;
    const long long n = vec ? F / 4 : F;
    dim3 grid((unsigned)((n + kAggThreads - 1) / kAggThreads), K);
    if (vec)
        scatter_mean_kernel<true><<<grid, kAggThreads, 0, s>>>(feats, F, d_order, d_offs, d_scale, agg);
    else
        scatter_mean_kernel<false><<<grid, kAggThreads, 0, s>>>(feats, F, d_order, d_offs, d_scale, agg);
    if (kf_ids_host) std::copy(ids.begin(), ids.end(), kf_ids_host);
    if (K_out) *K_out = K;
    return dc_check_launch(ctx, "scatter_mean_kernel");
}

// ---- row gather (the update step's per-edge input loads) -------------------
//
// Replaces the per-edge cudaMemcpy loop of main.cu:2215-2224 that loads
// batch_inps[e] = inps[ii[bs + e]] (one synchronous device-to-device copy per
// edge): dst[e] = src[idx[e]] for rows of F floats, one launch, float4
// streaming loads and stores.  Rows whose index is outside [0, num_rows) are
// written as zeros.
namespace {

template <bool kVec>
__global__ void __launch_bounds__(kAggThreads) gather_rows_kernel(
    const float* __restrict__ src, long long F, int num_rows, const int* __restrict__ idx,
    float* __restrict__ dst) {
    const int e = blockIdx.y;
    const int r = __ldg(idx + e);
    const bool ok = r >= 0 && r < num_rows;
    const long long stride = (long long)gridDim.x * kAggThreads;
    if (kVec) {
        const float4* s = reinterpret_cast<const float4*>(src + (size_t)(ok ? r : 0) * F);
        float4* d = reinterpret_cast<float4*>(dst + (size_t)e * F);
        for (long long i = (long long)blockIdx.x * kAggThreads + threadIdx.x; i < F / 4; i += stride)
            __stcs(d + i, ok ? __ldcs(s + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f));
    } else {
        const float* s = src + (size_t)(ok ? r : 0) * F;
        float* d = dst + (size_t)e * F;
        for (long long i = (long long)blockIdx.x * kAggThreads + threadIdx.x; i < F; i += stride)
            d[i] = ok ? __ldcs(s + i) : 0.0f;
    }
}

}  // namespace

int dc_gather_rows_impl(dc_ctx* ctx, const float* src, long long F, int num_rows, const int* idx,
                        int n, float* dst, cudaStream_t s) {
    const bool vec = (F % 4) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
    const long long work = vec ? F / 4 : F;
    long long bx = (work + kAggThreads * 4 - 1) / (kAggThreads * 4);  // ~4 items per thread
    if (bx < 1) bx = 1;
    if (bx > 65535) bx = 65535;
    dim3 grid((unsigned)bx, n);
    if (vec)
        gather_rows_kernel<true><<<grid, kAggThreads, 0, s>>>(src, F, num_rows, idx, dst);
    else
        gather_rows_kernel<false><<<grid, kAggThreads, 0, s>>>(src, F, num_rows, idx, dst);
    return dc_check_launch(ctx, "gather_rows_kernel");
}

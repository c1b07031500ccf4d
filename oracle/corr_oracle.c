/*
 * corr_oracle.c -- CPU restatement of the slam-hands DROID-SLAM correlation path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA library in
 * slam_hands_b200/csrc; it is never linked into, loaded by, or called from the
 * product path.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline legs may use it.
 *
 * Every function restates the arithmetic of the reference (paths relative to
 * the slam-hands project root):
 *
 *   orc_volume_*        cublasGemmBatchedEx / cublasGemmEx call in
 *                       cuda_slam/main.cu:1508-1515 and :1573-1581:
 *                       V[p][q] = alpha * sum_c f_ii[c][p] * f_jj[c][q]
 *                       (row-major [source pixel p][target pixel q]).
 *   orc_pool2x2         avg_pool_2x2_kernel, cuda_slam/main.cu:1150-1170
 *                       (and the cuDNN pooling of cuda_slam/nn.cuh:389-410):
 *                       out = 0.25f * (((a + b) + c) + d), floor on odd dims.
 *   orc_lookup          batch_corr_sample_kernel, cuda_slam/main.cu:1175-1217
 *                       (mode ORC_LOOKUP_BATCHED: nvcc contracts `out += s*wx*wy`
 *                       into fmaf(s*wx, wy, out)) and corr_index_kernel,
 *                       cuda_slam/main.cu:1079-1114 (mode ORC_LOOKUP_SINGLE:
 *                       atomicAdd of the rounded product s*wx*wy).
 *   orc_alt_lookup      no reference kernel exists.  It restates the lookup on
 *                       volumes V_l = alpha * <f_ii[:,p], P_l f_jj[:,q]>, which
 *                       equals pooling the volume over the target axes because
 *                       pooling is linear; dot products in double.
 *   orc_cpu_*           the fp32 C/OpenMP CPU baseline of
 *                       CudaDroid::batch_build_and_sample_correlation,
 *                       cuda_slam/main.cu:1555-1613.
 *
 * Compile with -ffp-contract=off: every fused multiply-add here is an explicit
 * fmaf() so that the order of rounding is the one stated in the comments.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_LOOKUP_BATCHED 0
#define ORC_LOOKUP_SINGLE 1

int orc_version(void) { return 1; }

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ------------------------------------------------------------------------ */
/* Volume build                                                              */
/* ------------------------------------------------------------------------ */

/* fp64 accumulation, alpha applied in double, rounded once to fp32.
 * fi, fj: [C][hw] channel-major (DroidState::fmaps slot layout, main.cu:677).
 * V: [hw][hw].  Golden reference for every precision mode (inputs are
 * pre-rounded to fp16/bf16/tf32 by the caller where a mode needs it). */
void orc_volume_f64(const float* fi, const float* fj, int C, int hw, double alpha,
                    float* V) {
    double* acc = (double*)malloc(sizeof(double) * (size_t)hw);
    for (int p = 0; p < hw; p++) {
        for (int q = 0; q < hw; q++) acc[q] = 0.0;
        for (int c = 0; c < C; c++) {
            double a = (double)fi[(size_t)c * hw + p];
            const float* b = fj + (size_t)c * hw;
            for (int q = 0; q < hw; q++) acc[q] += a * (double)b[q];
        }
        for (int q = 0; q < hw; q++) V[(size_t)p * hw + q] = (float)(alpha * acc[q]);
    }
    free(acc);
}

/* fp32 with the accumulation order of the library's exact-FFMA build kernel:
 * acc = 0; for c = 0..C-1: acc = fmaf(fi[c][p], fj[c][q], acc); V = alpha*acc. */
void orc_volume_f32_chain(const float* fi, const float* fj, int C, int hw, float alpha,
                          float* V) {
    float* acc = (float*)malloc(sizeof(float) * (size_t)hw);
    for (int p = 0; p < hw; p++) {
        for (int q = 0; q < hw; q++) acc[q] = 0.0f;
        for (int c = 0; c < C; c++) {
            float a = fi[(size_t)c * hw + p];
            const float* b = fj + (size_t)c * hw;
            for (int q = 0; q < hw; q++) acc[q] = fmaf(a, b[q], acc[q]);
        }
        for (int q = 0; q < hw; q++) V[(size_t)p * hw + q] = alpha * acc[q];
    }
    free(acc);
}

/* ------------------------------------------------------------------------ */
/* Pooling                                                                   */
/* ------------------------------------------------------------------------ */

/* in [N][H][W] -> out [N][H/2][W/2]; main.cu:1150-1170. */
void orc_pool2x2(const float* in, float* out, long long N, int H, int W) {
    int oH = H / 2, oW = W / 2;
    for (long long n = 0; n < N; n++) {
        const float* src = in + (size_t)n * H * W;
        float* dst = out + (size_t)n * oH * oW;
        for (int oy = 0; oy < oH; oy++)
            for (int ox = 0; ox < oW; ox++) {
                int iy = 2 * oy, ix = 2 * ox;
                float s = src[iy * W + ix] + src[iy * W + ix + 1];
                s = s + src[(iy + 1) * W + ix];
                s = s + src[(iy + 1) * W + ix + 1];
                dst[oy * oW + ox] = 0.25f * s;
            }
    }
}

/* ------------------------------------------------------------------------ */
/* Lookup                                                                    */
/* ------------------------------------------------------------------------ */

/* One (edge, level) of the lookup.  vol: [hw][Hl][Wl] for this edge and level;
 * coords: [2][h][w] (ch0 x, ch1 y, level-0 target pixels); out: this level's
 * D*D channel block, [D*D][h*w].  Channel (a*D + b): a = x offset, b = y offset
 * (main.cu:1203-1213).  The four contributions to output (a, b) arrive in the
 * reference loop order (i outer, j inner): taps (a,b), (a,b+1), (a+1,b),
 * (a+1,b+1), each weighted by (s*wx)*wy; out-of-bounds taps add nothing. */
static void lookup_level_range(const float* vol, const float* coords, float* out, int h,
                               int w, int Hl, int Wl, int r, float scale, int mode, int p0,
                               int p1) {
    int hw = h * w, D = 2 * r + 1;
    for (int p = p0; p < p1; p++) {
        float x0 = coords[p] * scale;
        float y0 = coords[hw + p] * scale;
        float fx = floorf(x0), fy = floorf(y0);
        float dx = x0 - fx, dy = y0 - fy;
        int bx = (int)fx - r, by = (int)fy - r;
        const float* row = vol + (size_t)p * Hl * Wl;
        float acc[64 * 64];
        for (int k = 0; k < D * D; k++) acc[k] = 0.0f;
        for (int i = 0; i < D + 1; i++) {
            for (int j = 0; j < D + 1; j++) {
                int x1 = bx + i, y1 = by + j;
                if (!(y1 >= 0 && y1 < Hl && x1 >= 0 && x1 < Wl)) continue;
                float s = row[y1 * Wl + x1];
                if (mode == ORC_LOOKUP_BATCHED) {
                    if (i > 0 && j > 0) acc[(i - 1) * D + (j - 1)] = fmaf(s * dx, dy, acc[(i - 1) * D + (j - 1)]);
                    if (i > 0 && j < D) acc[(i - 1) * D + j] = fmaf(s * dx, 1.0f - dy, acc[(i - 1) * D + j]);
                    if (i < D && j > 0) acc[i * D + (j - 1)] = fmaf(s * (1.0f - dx), dy, acc[i * D + (j - 1)]);
                    if (i < D && j < D) acc[i * D + j] = fmaf(s * (1.0f - dx), 1.0f - dy, acc[i * D + j]);
                } else {
                    if (i > 0 && j > 0) acc[(i - 1) * D + (j - 1)] += (s * dx) * dy;
                    if (i > 0 && j < D) acc[(i - 1) * D + j] += (s * dx) * (1.0f - dy);
                    if (i < D && j > 0) acc[i * D + (j - 1)] += (s * (1.0f - dx)) * dy;
                    if (i < D && j < D) acc[i * D + j] += (s * (1.0f - dx)) * (1.0f - dy);
                }
            }
        }
        for (int k = 0; k < D * D; k++) out[(size_t)k * hw + p] = acc[k];
    }
}

static void lookup_level(const float* vol, const float* coords, float* out, int h, int w,
                         int Hl, int Wl, int r, float scale, int mode) {
    lookup_level_range(vol, coords, out, h, w, Hl, Wl, r, scale, mode, 0, h * w);
}

/* levels[l]: [M][hw][h>>l][w>>l]; coords [M][2][h][w]; out [M][L*D*D][h][w].
 * Radius r <= 31.  Level l scales coordinates by 2^-l (main.cu:1189-1190). */
int orc_lookup(const float* const* levels, int L, const float* coords, float* out, int M,
               int h, int w, int r, int mode) {
    if (r < 0 || r > 31 || L < 1) return 1;
    int hw = h * w, D = 2 * r + 1;
    for (int e = 0; e < M; e++) {
        for (int l = 0; l < L; l++) {
            int Hl = h >> l, Wl = w >> l;
            const float* vol = levels[l] + (size_t)e * hw * Hl * Wl;
            lookup_level(vol, coords + (size_t)e * 2 * hw,
                         out + ((size_t)e * L * D * D + (size_t)l * D * D) * hw, h, w, Hl,
                         Wl, r, 1.0f / (float)(1 << l), mode);
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Feature-map pyramid and alt-corr (no reference kernel)                    */
/* ------------------------------------------------------------------------ */

/* fmap [C][H][W] -> [C][H/2][W/2], the same 2x2 average as orc_pool2x2. */
void orc_pool_fmap(const float* in, float* out, int C, int H, int W) {
    orc_pool2x2(in, out, C, H, W);
}

/* Alt-corr lookup for one edge.  fi: source fmap [C][hw]; pyr[l]: target fmap
 * pooled l times, [C][Hl*Wl] (pyr[0] = target fmap).  V_l[p][q] =
 * (float)(alpha * sum_c fi[c][p] * pyr[l][c][q]) in double, then the batched
 * lookup arithmetic of orc_lookup.  out: [L*D*D][h*w]. */
int orc_alt_lookup_edge(const float* fi, const float* const* pyr, int L, int C,
                        const float* coords, float* out, int h, int w, int r,
                        double alpha) {
    if (r < 0 || r > 31 || L < 1) return 1;
    int hw = h * w, D = 2 * r + 1;
    for (int l = 0; l < L; l++) {
        int Hl = h >> l, Wl = w >> l;
        float scale = 1.0f / (float)(1 << l);
        float* o = out + (size_t)l * D * D * hw;
        for (int p = 0; p < hw; p++) {
            float x0 = coords[p] * scale;
            float y0 = coords[hw + p] * scale;
            float fx = floorf(x0), fy = floorf(y0);
            float dx = x0 - fx, dy = y0 - fy;
            int bx = (int)fx - r, by = (int)fy - r;
            float acc[64 * 64];
            for (int k = 0; k < D * D; k++) acc[k] = 0.0f;
            for (int i = 0; i < D + 1; i++)
                for (int j = 0; j < D + 1; j++) {
                    int x1 = bx + i, y1 = by + j;
                    if (!(y1 >= 0 && y1 < Hl && x1 >= 0 && x1 < Wl)) continue;
                    double d = 0.0;
                    int q = y1 * Wl + x1;
                    for (int c = 0; c < C; c++)
                        d += (double)fi[(size_t)c * hw + p] * (double)pyr[l][(size_t)c * Hl * Wl + q];
                    float s = (float)(alpha * d);
                    if (i > 0 && j > 0) acc[(i - 1) * D + (j - 1)] = fmaf(s * dx, dy, acc[(i - 1) * D + (j - 1)]);
                    if (i > 0 && j < D) acc[(i - 1) * D + j] = fmaf(s * dx, 1.0f - dy, acc[(i - 1) * D + j]);
                    if (i < D && j > 0) acc[i * D + (j - 1)] = fmaf(s * (1.0f - dx), dy, acc[i * D + (j - 1)]);
                    if (i < D && j < D) acc[i * D + j] = fmaf(s * (1.0f - dx), 1.0f - dy, acc[i * D + j]);
                }
            for (int k = 0; k < D * D; k++) o[(size_t)k * hw + p] = acc[k];
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* CPU baseline: fp32 C/OpenMP build + pyramid + lookup per edge             */
/* ------------------------------------------------------------------------ */

/* fmaps [K][C][hw] fp32; ii/jj host edge lists; coords [M][2][hw];
 * out [M][L*D*D][hw].  work: caller-provided scratch of
 * orc_cpu_work_floats(h, w, L) floats.  Parallel over source-pixel blocks
 * with nthreads OpenMP threads (<=0: all). */
long long orc_cpu_work_floats(int h, int w, int L) {
    long long hw = (long long)h * w, n = 0;
    for (int l = 0; l < L; l++) n += hw * (long long)(h >> l) * (w >> l);
    return n;
}

int orc_cpu_build_and_sample(const float* fmaps, int C, int h, int w, const int* ii,
                             const int* jj, int M, const float* coords, float* out,
                             int L, int r, float alpha, float* work, int nthreads) {
    if (L < 1 || L > 8 || r < 0 || r > 31) return 1;
    int hw = h * w, D = 2 * r + 1;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#else
    nthreads = 1;
#endif
    float* lev[8];
    lev[0] = work;
    for (int l = 1; l < L; l++)
        lev[l] = lev[l - 1] + (size_t)hw * (h >> (l - 1)) * (w >> (l - 1));
    for (int e = 0; e < M; e++) {
        const float* fi = fmaps + (size_t)ii[e] * C * hw;
        const float* fj = fmaps + (size_t)jj[e] * C * hw;
        float* V = lev[0];
        /* cache-blocked fp32 GEMM: 8 source rows x 512 targets per block */
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads)
        for (int pb = 0; pb < hw; pb += 8) {
            int pe = pb + 8 < hw ? pb + 8 : hw;
            for (int qb = 0; qb < hw; qb += 512) {
                int qe = qb + 512 < hw ? qb + 512 : hw;
                float acc[8][512];
                for (int p = pb; p < pe; p++)
                    for (int q = qb; q < qe; q++) acc[p - pb][q - qb] = 0.0f;
                for (int c = 0; c < C; c++) {
                    const float* b = fj + (size_t)c * hw;
                    for (int p = pb; p < pe; p++) {
                        float a = fi[(size_t)c * hw + p];
                        float* ar = acc[p - pb];
                        for (int q = qb; q < qe; q++) ar[q - qb] = fmaf(a, b[q], ar[q - qb]);
                    }
                }
                for (int p = pb; p < pe; p++)
                    for (int q = qb; q < qe; q++)
                        V[(size_t)p * hw + q] = alpha * acc[p - pb][q - qb];
            }
        }
        for (int l = 1; l < L; l++) {
            int H = h >> (l - 1), W = w >> (l - 1);
#pragma omp parallel for schedule(static) num_threads(nthreads)
            for (int p = 0; p < hw; p++)
                orc_pool2x2(lev[l - 1] + (size_t)p * H * W, lev[l] + (size_t)p * (H / 2) * (W / 2), 1, H, W);
        }
        const float* ce = coords + (size_t)e * 2 * hw;
        float* oe = out + (size_t)e * L * D * D * hw;
#pragma omp parallel for schedule(static) num_threads(nthreads)
        for (int pb = 0; pb < hw; pb += 64) {
            int pe = pb + 64 < hw ? pb + 64 : hw;
            for (int l = 0; l < L; l++)
                lookup_level_range(lev[l], ce, oe + (size_t)l * D * D * hw, h, w, h >> l,
                                   w >> l, r, 1.0f / (float)(1 << l), ORC_LOOKUP_BATCHED,
                                   pb, pe);
        }
    }
    return 0;
}

/* GraphAgg scatter_mean (cuda_slam/main.cu:2255-2294) as the reference runs it:
 * compact keyframe index = rank of ii[e] among the distinct ii in ascending
 * order (std::set); the compact buffer starts at 0 (cudaMemset, :2269); every
 * edge e in order adds its features with scale_add_kernel(dst, src, 1.0f)
 * (nn.cuh:382-385: dst += scale * src, contracted by nvcc to fmaf(scale, src,
 * dst)); then keyframes with count > 1 get scale_add_kernel(dst, dst,
 * 1.0f / count - 1.0f) (:2287-2294), i.e. fmaf(s, dst, dst).
 * feats [E][F] -> agg [K][F]; ids [K]; returns K. */
int orc_scatter_mean(const float* feats, long long F, const int* ii, int E, float* agg, int* ids) {
    int K = 0;
    for (int e = 0; e < E; e++) {  /* distinct ids, ascending (insertion sort) */
        int v = ii[e], pos = 0, dup = 0;
        while (pos < K && ids[pos] < v) pos++;
        if (pos < K && ids[pos] == v) dup = 1;
        if (!dup) {
            for (int m = K; m > pos; m--) ids[m] = ids[m - 1];
            ids[pos] = v;
            K++;
        }
    }
    for (long long i = 0; i < (long long)K * F; i++) agg[i] = 0.0f;
    int* count = (int*)calloc(K > 0 ? K : 1, sizeof(int));
    for (int e = 0; e < E; e++) {
        int k = 0;
        while (ids[k] != ii[e]) k++;
        float* dst = agg + (size_t)k * F;
        const float* src = feats + (size_t)e * F;
        for (long long i = 0; i < F; i++) dst[i] = fmaf(1.0f, src[i], dst[i]);
        count[k]++;
    }
    for (int k = 0; k < K; k++) {
        if (count[k] > 1) {
            float s = 1.0f / (float)count[k] - 1.0f;
            float* dst = agg + (size_t)k * F;
            for (long long i = 0; i < F; i++) dst[i] = fmaf(s, dst[i], dst[i]);
        }
    }
    free(count);
    return K;
}

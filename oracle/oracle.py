"""numpy front end of the CPU oracle (liboracle.so, built from corr_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA library, never the thing
measured or shipped.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline legs import this module.

Each function mirrors one restatement in corr_oracle.c; the reference lines it
follows are cited there (cuda_slam/main.cu:1079-1217, :1499-1613,
cuda_slam/nn.cuh:389-410).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

LOOKUP_BATCHED = 0  # batch_corr_sample_kernel arithmetic (main.cu:1175-1217)
LOOKUP_SINGLE = 1   # corr_index_kernel arithmetic (main.cu:1079-1114)

_fp = ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int)


def build() -> str:
    """Compile liboracle.so with the committed Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_volume_f64.argtypes = [_fp, _fp, ctypes.c_int, ctypes.c_int, ctypes.c_double, _fp]
        L.orc_volume_f32_chain.argtypes = [_fp, _fp, ctypes.c_int, ctypes.c_int, ctypes.c_float, _fp]
        L.orc_pool2x2.argtypes = [_fp, _fp, ctypes.c_longlong, ctypes.c_int, ctypes.c_int]
        L.orc_lookup.argtypes = [ctypes.POINTER(_fp), ctypes.c_int, _fp, _fp, ctypes.c_int,
                                 ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_alt_lookup_edge.argtypes = [_fp, ctypes.POINTER(_fp), ctypes.c_int, ctypes.c_int,
                                          _fp, _fp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_double]
        L.orc_cpu_work_floats.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_cpu_work_floats.restype = ctypes.c_longlong
        L.orc_cpu_build_and_sample.argtypes = [_fp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                               _ip, _ip, ctypes.c_int, _fp, _fp, ctypes.c_int,
                                               ctypes.c_int, ctypes.c_float, _fp, ctypes.c_int]
        L.orc_scatter_mean.argtypes = [_fp, ctypes.c_longlong, _ip, ctypes.c_int, _fp, _ip]
        L.orc_scatter_mean.restype = ctypes.c_int
        _lib = L
    return _lib


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_fp)


def _i(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_ip)


def volume_f64(fi: np.ndarray, fj: np.ndarray, alpha: float) -> np.ndarray:
    """V[p][q] = alpha * sum_c fi[c][p] fj[c][q], fp64 accumulate. fi, fj: [C][h][w]."""
    C = fi.shape[0]
    hw = fi.size // C
    fi = np.ascontiguousarray(fi, np.float32).reshape(C, hw)
    fj = np.ascontiguousarray(fj, np.float32).reshape(C, hw)
    V = np.empty((hw, hw), np.float32)
    lib().orc_volume_f64(_f(fi), _f(fj), C, hw, float(alpha), _f(V))
    return V


def volume_f32_chain(fi: np.ndarray, fj: np.ndarray, alpha: float) -> np.ndarray:
    """fp32 volume with a sequential fmaf chain over channels, then alpha*acc."""
    C = fi.shape[0]
    hw = fi.size // C
    fi = np.ascontiguousarray(fi, np.float32).reshape(C, hw)
    fj = np.ascontiguousarray(fj, np.float32).reshape(C, hw)
    V = np.empty((hw, hw), np.float32)
    lib().orc_volume_f32_chain(_f(fi), _f(fj), C, hw, np.float32(alpha), _f(V))
    return V


def pool2x2(x: np.ndarray) -> np.ndarray:
    """avg_pool_2x2_kernel over the last two dims (floor on odd dims)."""
    x = np.ascontiguousarray(x, np.float32)
    H, W = x.shape[-2:]
    N = x.size // (H * W)
    out = np.empty(x.shape[:-2] + (H // 2, W // 2), np.float32)
    lib().orc_pool2x2(_f(x), _f(out), N, H, W)
    return out


def pyramid(V0: np.ndarray, h: int, w: int, levels: int = 4) -> list:
    """Cascaded pyramid of a volume [..., hw, hw] -> list of [..., hw, h>>l, w>>l]."""
    lead = V0.shape[:-1]
    out = [np.ascontiguousarray(V0, np.float32).reshape(lead + (h, w))]
    for _ in range(1, levels):
        out.append(pool2x2(out[-1]))
    return out


def lookup(levels: list, coords: np.ndarray, h: int, w: int, radius: int = 3,
           mode: int = LOOKUP_BATCHED) -> np.ndarray:
    """levels[l]: [M, hw, h>>l, w>>l]; coords [M, 2, h, w] -> out [M, L*D*D, h, w]."""
    M = coords.shape[0]
    L = len(levels)
    D = 2 * radius + 1
    levs = [np.ascontiguousarray(v, np.float32) for v in levels]
    for l, v in enumerate(levs):
        assert v.size == M * h * w * (h >> l) * (w >> l), (l, v.shape)
    coords = np.ascontiguousarray(coords, np.float32)
    out = np.empty((M, L * D * D, h, w), np.float32)
    arr = (_fp * L)(*[_f(v) for v in levs])
    rc = lib().orc_lookup(arr, L, _f(coords), _f(out), M, h, w, radius, mode)
    assert rc == 0
    return out


def fmap_pyramid(f: np.ndarray, levels: int = 4) -> list:
    """fmap [C, h, w] -> [P_0 f, ..., P_{L-1} f], P = cascaded 2x2 average."""
    out = [np.ascontiguousarray(f, np.float32)]
    for _ in range(1, levels):
        out.append(pool2x2(out[-1]))
    return out


def alt_lookup_edge(fi: np.ndarray, fj: np.ndarray, coords: np.ndarray, alpha: float,
                    radius: int = 3, levels: int = 4) -> np.ndarray:
    """On-the-fly lookup for one edge. fi, fj [C,h,w]; coords [2,h,w] -> [L*D*D, h, w]."""
    C, h, w = fi.shape
    D = 2 * radius + 1
    pyr = fmap_pyramid(fj, levels)
    pyr = [np.ascontiguousarray(p.reshape(C, -1)) for p in pyr]
    fi = np.ascontiguousarray(fi, np.float32).reshape(C, h * w)
    coords = np.ascontiguousarray(coords, np.float32)
    out = np.empty((levels * D * D, h, w), np.float32)
    arr = (_fp * levels)(*[_f(p) for p in pyr])
    rc = lib().orc_alt_lookup_edge(_f(fi), arr, levels, C, _f(coords), _f(out), h, w, radius,
                                   float(alpha))
    assert rc == 0
    return out


def cpu_build_and_sample(fmaps: np.ndarray, ii: np.ndarray, jj: np.ndarray,
                         coords: np.ndarray, alpha: float, radius: int = 3,
                         levels: int = 4, threads: int = 0) -> np.ndarray:
    """fp32 C/OpenMP baseline of batch_build_and_sample_correlation.

    fmaps [K, C, h, w]; ii, jj [M] int; coords [M, 2, h, w] -> [M, L*D*D, h, w]."""
    K, C, h, w = fmaps.shape
    M = len(ii)
    D = 2 * radius + 1
    fmaps = np.ascontiguousarray(fmaps, np.float32)
    ii = np.ascontiguousarray(ii, np.int32)
    jj = np.ascontiguousarray(jj, np.int32)
    coords = np.ascontiguousarray(coords, np.float32)
    out = np.empty((M, levels * D * D, h, w), np.float32)
    work = np.empty(lib().orc_cpu_work_floats(h, w, levels), np.float32)
    rc = lib().orc_cpu_build_and_sample(_f(fmaps), C, h, w, _i(ii), _i(jj), M, _f(coords),
                                        _f(out), levels, radius, np.float32(alpha), _f(work),
                                        int(threads))
    assert rc == 0
    return out


def max_threads() -> int:
    return int(lib().orc_max_threads())


# ---------------------------------------------------------------- reprojection

def _rotate(q: np.ndarray, X: np.ndarray) -> np.ndarray:
    """q X q* in the form of actSO3 (cuda_slam/se3.cuh:8-17): uv = 2 q x X,
    Y = X + w uv + q x uv.  q = (x, y, z, w); X [..., 3]."""
    qv, w = q[:3], q[3]
    uv = 2.0 * np.cross(qv, X)
    return X + w * uv + np.cross(qv, uv)


def relative_pose(pi: np.ndarray, pj: np.ndarray):
    """G_ij = G_j G_i^-1 for poses (t, q) [7] (relSE3, cuda_slam/se3.cuh:44-55)."""
    ti, qi, tj, qj = pi[:3], pi[3:], pj[:3], pj[3:]
    qij = np.array([
        -qj[3] * qi[0] + qj[0] * qi[3] - qj[1] * qi[2] + qj[2] * qi[1],
        -qj[3] * qi[1] + qj[1] * qi[3] - qj[2] * qi[0] + qj[0] * qi[2],
        -qj[3] * qi[2] + qj[2] * qi[3] - qj[0] * qi[1] + qj[1] * qi[0],
        qj[3] * qi[3] + qj[0] * qi[0] + qj[1] * qi[1] + qj[2] * qi[2]])
    tij = tj - _rotate(qij, ti)
    return tij, qij


def project(poses: np.ndarray, disps: np.ndarray, intrinsics: np.ndarray, ii, jj):
    """float64 restatement of projmap_kernel (cuda_slam/se3.cuh:118-177) with the
    output in the lookup's layout (batch_coords_hw2_to_2hw, main.cu:1135-1146).
    poses [N, 7], disps [N, H, W], intrinsics (fx, fy, cx, cy).  Returns
    (coords [M, 2, H, W], valid [M, H, W]); an edge with ii/jj outside [0, N)
    keeps the pixel grid and is not valid."""
    poses = np.asarray(poses, np.float64)
    disps = np.asarray(disps, np.float64)
    fx, fy, cx, cy = (float(v) for v in intrinsics)
    N, H, W = disps.shape
    v, u = np.meshgrid(np.arange(H, dtype=np.float64), np.arange(W, dtype=np.float64),
                       indexing="ij")
    M = len(ii)
    coords = np.empty((M, 2, H, W))
    valid = np.zeros((M, H, W))
    for e, (i, j) in enumerate(zip(ii, jj)):
        if not (0 <= i < N and 0 <= j < N):
            coords[e, 0], coords[e, 1] = u, v
            continue
        tij, qij = relative_pose(poses[i], poses[j])
        Xi = np.stack([(u - cx) / fx, (v - cy) / fy, np.ones_like(u)], -1)
        Xj = _rotate(qij, Xi) + disps[i][..., None] * tij
        z = Xj[..., 2]
        front = z > 0.01
        zs = np.where(front, z, 1.0)
        coords[e, 0] = np.where(front, fx * (Xj[..., 0] / zs) + cx, u)
        coords[e, 1] = np.where(front, fy * (Xj[..., 1] / zs) + cy, v)
        valid[e] = (z > 0.25).astype(np.float64)
    return coords, valid



def scatter_mean(feats: np.ndarray, ii) -> tuple:
    """GraphAgg scatter_mean as the reference computes it (orc_scatter_mean,
    cuda_slam/main.cu:2255-2294).  feats [E, ...] float32 -> (agg [K, ...], ids [K])."""
    feats = np.ascontiguousarray(feats, np.float32)
    ii = np.ascontiguousarray(ii, np.int32)
    E = feats.shape[0]
    F = int(np.prod(feats.shape[1:]))
    agg = np.empty((E, F), np.float32)
    ids = np.empty(E, np.int32)
    K = lib().orc_scatter_mean(_f(feats), F, _i(ii), E, _f(agg), _i(ids))
    return agg[:K].reshape((K,) + feats.shape[1:]), ids[:K].copy()


def corr_encode(corr: np.ndarray, weight: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """The update operator's first correlation-encoder layer as the reference
    computes it: a 1x1 convolution 196 -> 128 with bias (UpdateModule corr_enc_0,
    cuda_slam/main.cu:552-553), relu_inplace, round_to_fp16 (main.cu:603-606).
    Here in float64 before the final ReLU and fp16 rounding.
    corr [M, ci, h, w], weight [co, ci] (or [co, ci, 1, 1]), bias [co]
    -> [M, co, h, w] float16."""
    w = np.asarray(weight, np.float64).reshape(weight.shape[0], -1)
    x = np.asarray(corr, np.float64)
    y = np.einsum("oc,mchw->mohw", w, x) + np.asarray(bias, np.float64)[None, :, None, None]
    return np.maximum(y, 0.0).astype(np.float16)

"""numpy front end of oracle/_ref/libref.so: the reference's own correlation
kernels (cuda_slam/main.cu:1077-1217, extracted at build time, never committed)
driven like CudaDroid (main.cu:1529-1613) on a GPU.

TEST INFRASTRUCTURE ONLY: the second checker, run on the GPU box.  The library
is built here by `make -C oracle ref` (needs the read-only reference tree) and
travels to the GPU box prebuilt; available() is False where it is missing.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libref.so")
_fp = ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int)
_lib = None


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(LIB_PATH)
        L.ref_pool.argtypes = [_fp, _fp, ctypes.c_longlong, ctypes.c_int, ctypes.c_int]
        L.ref_lookup_batched.argtypes = [ctypes.POINTER(_fp), _fp, _fp, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int]
        L.ref_lookup_single.argtypes = [ctypes.POINTER(_fp), _fp, _fp, ctypes.c_int,
                                        ctypes.c_int]
        L.ref_build_and_sample_fp16.argtypes = [_fp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                _ip, _ip, ctypes.c_int, _fp, ctypes.c_float,
                                                _fp, _fp, ctypes.c_int, _fp]
        L.ref_project.argtypes = [_fp, _fp, _fp, ctypes.c_int, _ip, _ip, ctypes.c_int,
                                  ctypes.c_int, ctypes.c_int, _fp, _fp]
        L.ref_scatter_mean.argtypes = [_fp, ctypes.c_longlong, _ip, ctypes.c_int, _fp, _ip]
        _lib = L
    return _lib


def project(poses, disps, intrinsics, ii, jj):
    """The reference's projmap_kernel + batch_coords_hw2_to_2hw on the GPU
    (se3.cuh:118-177, main.cu:1135-1146).  Returns (coords [M,2,H,W], valid [M,H,W])."""
    poses = np.ascontiguousarray(poses, np.float32)
    disps = np.ascontiguousarray(disps, np.float32)
    intr = np.ascontiguousarray(intrinsics, np.float32)
    ii = np.ascontiguousarray(ii, np.int32)
    jj = np.ascontiguousarray(jj, np.int32)
    N, H, W = disps.shape
    M = len(ii)
    coords = np.empty((M, 2, H, W), np.float32)
    valid = np.empty((M, H, W), np.float32)
    rc = lib().ref_project(_f(poses), _f(disps), _f(intr), N, ii.ctypes.data_as(_ip),
                           jj.ctypes.data_as(_ip), M, H, W, _f(coords), _f(valid))
    assert rc == 0, rc
    return coords, valid


def _f(a):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_fp)


def pool(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    H, W = x.shape[-2:]
    out = np.empty(x.shape[:-2] + (H // 2, W // 2), np.float32)
    assert lib().ref_pool(_f(x), _f(out), x.size // (H * W), H, W) == 0
    return out


def lookup_batched(levels, coords, h, w):
    levs = [np.ascontiguousarray(v, np.float32) for v in levels]
    coords = np.ascontiguousarray(coords, np.float32)
    M = coords.shape[0]
    out = np.empty((M, 196, h, w), np.float32)
    arr = (_fp * 4)(*[_f(v) for v in levs])
    assert lib().ref_lookup_batched(arr, _f(coords), _f(out), M, h, w) == 0
    return out


def lookup_single(levels, coords, h, w):
    levs = [np.ascontiguousarray(v, np.float32) for v in levels]
    coords = np.ascontiguousarray(coords, np.float32)
    out = np.empty((196, h, w), np.float32)
    arr = (_fp * 4)(*[_f(v) for v in levs])
    assert lib().ref_lookup_single(arr, _f(coords), _f(out), h, w) == 0
    return out


def build_and_sample_fp16(fmaps, ii, jj, coords, alpha, want_vol0=False, iters=0):
    """Returns (out [M,196,h,w], vol0 or None, ms_per_pass or None)."""
    fmaps = np.ascontiguousarray(fmaps, np.float32)
    K, C, h, w = fmaps.shape
    assert C == 128
    ii = np.ascontiguousarray(ii, np.int32)
    jj = np.ascontiguousarray(jj, np.int32)
    coords = np.ascontiguousarray(coords, np.float32)
    M = len(ii)
    out = np.empty((M, 196, h, w), np.float32)
    vol0 = np.empty((M, h * w, h * w), np.float32) if want_vol0 else None
    ms = np.zeros(1, np.float32)
    rc = lib().ref_build_and_sample_fp16(
        _f(fmaps), K, h, w, ii.ctypes.data_as(_ip), jj.ctypes.data_as(_ip), M, _f(coords),
        float(alpha), _f(out), _f(vol0) if want_vol0 else None, int(iters), _f(ms))
    assert rc == 0
    return out, vol0, (float(ms[0]) if iters else None)


def scatter_mean(feats, ii):
    """The reference's GraphAgg loop on the GPU (memset, scale_add_kernel per edge
    and per keyframe, main.cu:2262-2294; nn.cuh:381-385).  feats [E, ...];
    returns (agg [K, ...], keyframe ids ascending)."""
    feats = np.ascontiguousarray(feats, np.float32)
    ii = np.ascontiguousarray(ii, np.int32)
    E = feats.shape[0]
    F = int(np.prod(feats.shape[1:]))
    ids = np.unique(ii)
    agg = np.empty((len(ids),) + feats.shape[1:], np.float32)
    K = ctypes.c_int(0)
    rc = lib().ref_scatter_mean(_f(feats), F, ii.ctypes.data_as(_ip), E, _f(agg), ctypes.byref(K))
    assert rc == 0 and K.value == len(ids), rc
    return agg, ids

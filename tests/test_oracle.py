"""CPU tests of the oracle: known-answer tests for the lookup, pooling and volume
semantics of the reference (cuda_slam/main.cu:1079-1217, :1499-1613), an
independent numpy restatement, and the linearity identity behind alt-corr."""
import math

import numpy as np
import pytest

from slam_hands_b200 import configs


def normwise(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def np_lookup_reference(vol_rows, coords, h, w, l, r=3):
    """Independent numpy restatement of one level of batch_corr_sample_kernel
    (main.cu:1175-1217) in float64: vol_rows [hw, Hl, Wl], coords [2, h, w]."""
    Hl, Wl = h >> l, w >> l
    D = 2 * r + 1
    x0 = coords[0].reshape(-1).astype(np.float32) * np.float32(2.0 ** -l)
    y0 = coords[1].reshape(-1).astype(np.float32) * np.float32(2.0 ** -l)
    fx, fy = np.floor(x0), np.floor(y0)
    dx, dy = (x0 - fx).astype(np.float64), (y0 - fy).astype(np.float64)
    out = np.zeros((D * D, h * w))
    for p in range(h * w):
        for i in range(D + 1):
            for j in range(D + 1):
                x1, y1 = int(fx[p]) - r + i, int(fy[p]) - r + j
                if not (0 <= x1 < Wl and 0 <= y1 < Hl):
                    continue
                s = float(vol_rows[p, y1, x1])
                if i > 0 and j > 0:
                    out[(i - 1) * D + (j - 1), p] += s * dx[p] * dy[p]
                if i > 0 and j < D:
                    out[(i - 1) * D + j, p] += s * dx[p] * (1 - dy[p])
                if i < D and j > 0:
                    out[i * D + (j - 1), p] += s * (1 - dx[p]) * dy[p]
                if i < D and j < D:
                    out[i * D + j, p] += s * (1 - dx[p]) * (1 - dy[p])
    return out.reshape(D * D, h, w)


def rand_setup(h, w, C=32, seed=0, sigma=2.0, M=1):
    rng = np.random.default_rng(seed)
    f = rng.standard_normal((M + 1, C, h, w), dtype=np.float32)
    coords = (configs.grid_coords(h, w)[None] + rng.normal(0, sigma, (M, 2, h, w))).astype(np.float32)
    return f, coords


def test_integer_coords_pin_channel_order(oracle):
    # KAT: integer coordinates -> out[a*7+b][p] = V[p][(y+b-3)*W + (x+a-3)], zero outside
    h, w = 6, 8
    rng = np.random.default_rng(1)
    V = rng.standard_normal((h * w, h * w)).astype(np.float32)
    coords = configs.grid_coords(h, w)[None]
    levs = oracle.pyramid(V[None], h, w, 1)
    out = oracle.lookup(levs, coords, h, w, 3)[0]
    for p in range(h * w):
        y, x = divmod(p, w)
        for a in range(7):
            for b in range(7):
                xx, yy = x + a - 3, y + b - 3
                exp = V[p, yy * w + xx] if (0 <= xx < w and 0 <= yy < h) else 0.0
                assert out[a * 7 + b, y, x] == exp


def test_constant_volume_border_weights(oracle):
    # KAT: constant volume of ones -> 1 where all four taps are inside, partial at borders
    h, w = 8, 8
    V = np.ones((1, h * w, h, w), np.float32)
    coords = np.full((1, 2, h, w), 4.25, np.float32)  # every pixel looks at (4.25, 4.25)
    out = oracle.lookup([V], coords, h, w, 3)[0]
    # window x taps floor(4.25)-3 .. +4 = 1..8 -> tap 8 is outside (W=8)
    # output a uses taps a and a+1: a = 0..6 -> taps 1..7 inside except a=6 (tap 8 out)
    inside = out[: 6 * 7].reshape(6, 7, h, w)[:, :6]
    assert np.allclose(inside, 1.0, atol=1e-6)
    edge = out[6 * 7 + 0]  # a = 6, b = 0: x tap 7 inside (weight 1-dx), tap 8 outside
    assert np.allclose(edge, 0.75, atol=1e-6)


def test_all_out_of_bounds_is_zero(oracle):
    h, w = 6, 8
    V = np.random.default_rng(2).standard_normal((1, h * w, h, w)).astype(np.float32)
    coords = np.full((1, 2, h, w), -100.0, np.float32)
    out = oracle.lookup([V], coords, h, w, 3)
    assert np.all(out == 0.0)
    coords = np.full((1, 2, h, w), 1000.0, np.float32)
    assert np.all(oracle.lookup([V], coords, h, w, 3) == 0.0)


def test_negative_fractional_floor(oracle):
    # floor(-0.5) = -1: window starts at -4, dx = 0.5
    h, w = 6, 8
    rng = np.random.default_rng(3)
    V = rng.standard_normal((1, h * w, h, w)).astype(np.float32)
    coords = np.zeros((1, 2, h, w), np.float32)
    coords[0, 0] = -0.5
    coords[0, 1] = 2.0
    out = oracle.lookup([V], coords, h, w, 3)[0]
    ref = np_lookup_reference(V[0], coords[0], h, w, 0)
    assert normwise(out, ref) < 1e-6
    # a = 3 (x offset 0): taps x = -1 (outside) and x = 0 (weight dx = 0.5)
    p = 0
    b = 3  # y offset 0 -> y tap 2 with weight 1
    assert out[3 * 7 + b, 0, 0] == pytest.approx(0.5 * V[0, p, 2, 0], rel=1e-6)


@pytest.mark.parametrize("h,w", [(6, 8), (5, 9), (41, 73)])
def test_pool_floor_odd_dims(oracle, h, w):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((3, h, w)).astype(np.float32)
    y = oracle.pool2x2(x)
    assert y.shape == (3, h // 2, w // 2)
    ref = 0.25 * (((x[:, 0:2 * (h // 2):2, 0:2 * (w // 2):2] + x[:, 0:2 * (h // 2):2, 1:2 * (w // 2):2])
                   + x[:, 1:2 * (h // 2):2, 0:2 * (w // 2):2]) + x[:, 1:2 * (h // 2):2, 1:2 * (w // 2):2])
    assert np.array_equal(y, ref.astype(np.float32))


def test_pyramid_shapes_41x73(oracle):
    h, w = 41, 73
    V = np.zeros((2, h * w), np.float32)
    levs = oracle.pyramid(V, h, w, 4)
    assert [lv.shape[-2:] for lv in levs] == [(41, 73), (20, 36), (10, 18), (5, 9)]


@pytest.mark.parametrize("h,w", [(6, 8), (5, 9), (12, 16)])
def test_lookup_matches_numpy_restatement(oracle, h, w):
    f, coords = rand_setup(h, w, seed=5)
    V = oracle.volume_f64(f[0], f[1], 1 / 16)
    levs = oracle.pyramid(V[None], h, w, 4 if min(h, w) >= 8 else 2)
    out = oracle.lookup(levs, coords, h, w, 3)[0]
    for l in range(len(levs)):
        ref = np_lookup_reference(levs[l][0], coords[0], h, w, l)
        assert normwise(out[l * 49:(l + 1) * 49], ref) < 2e-6


def test_single_vs_batched_arith_agree(oracle):
    h, w = 12, 16
    f, coords = rand_setup(h, w, seed=6)
    V = oracle.volume_f64(f[0], f[1], 1 / 16)
    levs = oracle.pyramid(V[None], h, w, 4)
    a = oracle.lookup(levs, coords, h, w, 3, oracle.LOOKUP_BATCHED)
    b = oracle.lookup(levs, coords, h, w, 3, oracle.LOOKUP_SINGLE)
    assert normwise(a, b) < 1e-6


def test_volume_orientation_and_alpha(oracle):
    # V[p][q] = alpha * <f_ii[:, p], f_jj[:, q]>  (A = fmaps[jj], B = fmaps[ii], main.cu:1560-1562)
    h, w, C = 4, 6, 32
    f, _ = rand_setup(h, w, C=C, seed=7)
    for alpha in (1 / 16, 1 / 128, 1 / math.sqrt(128)):
        V = oracle.volume_f64(f[0], f[1], alpha)
        ref = alpha * (f[0].reshape(C, -1).astype(np.float64).T @ f[1].reshape(C, -1).astype(np.float64))
        assert np.allclose(V, ref, rtol=1e-6, atol=1e-6)
        V32 = oracle.volume_f32_chain(f[0], f[1], alpha)
        assert normwise(V32, ref) < 1e-6


def test_alt_equals_materialised_by_linearity(oracle):
    # pooling the volume over target axes == correlating with pooled target maps
    h, w, C = 16, 24, 32
    f, coords = rand_setup(h, w, C=C, seed=8, sigma=4.0)
    alpha = 1 / math.sqrt(128)
    V = oracle.volume_f64(f[0], f[1], alpha)
    mat = oracle.lookup(oracle.pyramid(V[None], h, w, 4), coords, h, w, 3)[0]
    alt = oracle.alt_lookup_edge(f[0], f[1], coords[0], alpha, 3, 4)
    assert normwise(alt, mat) < 1e-5


def test_cpu_baseline_matches_oracle(oracle):
    h, w, C = 12, 16, 128
    rng = np.random.default_rng(9)
    fm = rng.standard_normal((3, C, h, w), dtype=np.float32)
    ii, jj = np.array([0, 2], np.int32), np.array([1, 0], np.int32)
    coords = (configs.grid_coords(h, w)[None] + rng.normal(0, 2, (2, 2, h, w))).astype(np.float32)
    out = oracle.cpu_build_and_sample(fm, ii, jj, coords, 1 / 16, threads=2)
    for e in range(2):
        V = oracle.volume_f64(fm[ii[e]], fm[jj[e]], 1 / 16)
        ref = oracle.lookup(oracle.pyramid(V[None], h, w, 4), coords[e:e + 1], h, w, 3)[0]
        assert normwise(out[e], ref) < 1e-5


def test_workload_edge_rules():
    # pair counts of the benchmark edge rules and the seeded subsets
    for name, n_pairs in [("C2", 60), ("C3", 1776), ("C4", 172), ("C5", 11688)]:
        wl = configs.WORKLOADS[name]
        assert len(configs.ordered_pairs(wl.frames, wl.max_offset)) == n_pairs
        ii, jj = configs.make_edges(wl)
        assert len(ii) == wl.edges
        assert len(set(zip(ii.tolist(), jj.tolist()))) == wl.edges
        d = np.abs(ii - jj)
        assert d.min() >= 1 and d.max() <= wl.max_offset

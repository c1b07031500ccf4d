"""Seeded synthetic workloads C1..C5 (the shapes, edge rules and coordinate
distributions of the benchmark configurations; there is no dataset).

  C1  48x64,  2 frames, 1 edge (0 -> 1), coords = grid + U(-4, 4), materialised
  C2  48x64, 12 frames, 48 of the 60 ordered pairs with 1 <= |i-j| <= 3,
      coords = grid + N(0, 2), materialised (the reference's frontend chunk,
      MAX_BATCH_EDGES = 48, cuda_slam/main.cu:1314)
  C3  48x64, 64 frames, 800 of the 1776 pairs with 1 <= |i-j| <= 16,
      coords = grid + N(0, 8), alt-corr
  C4  54x96, 24 frames, 96 of the 172 pairs with 1 <= |i-j| <= 4,
      coords = grid + N(0, 3), materialised
  C5  54x96, 256 frames, 2048 of the 11688 pairs with 1 <= |i-j| <= 24,
      coords = grid + N(0, 8), alt-corr, edges sharded over GPUs

Feature maps are i.i.d. N(0, 1) fp32, alpha = 1/sqrt(128).  Edge subsets are
drawn without replacement from the ordered pair list (i ascending, then j) with
numpy's default_rng(seed); the pair rule generates more pairs than the stated
edge count for C2 and C4, so the seeded subset is the stated count.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Workload:
    name: str
    h: int
    w: int
    frames: int
    max_offset: int
    edges: int
    coord_noise: str   # "uniform4" or "normal"
    sigma: float
    mode: str          # "materialised" or "alt"
    channels: int = 128
    alpha: float = 1.0 / math.sqrt(128.0)


WORKLOADS = {
    "C1": Workload("C1", 48, 64, 2, 1, 1, "uniform4", 4.0, "materialised"),
    "C2": Workload("C2", 48, 64, 12, 3, 48, "normal", 2.0, "materialised"),
    "C3": Workload("C3", 48, 64, 64, 16, 800, "normal", 8.0, "alt"),
    "C4": Workload("C4", 54, 96, 24, 4, 96, "normal", 3.0, "materialised"),
    "C5": Workload("C5", 54, 96, 256, 24, 2048, "normal", 8.0, "alt"),
}

SEED = 20261201


def ordered_pairs(frames: int, max_offset: int) -> np.ndarray:
    """All (i, j) with 1 <= |i - j| <= max_offset, i ascending then j ascending."""
    out = [(i, j) for i in range(frames) for j in range(frames)
           if i != j and abs(i - j) <= max_offset]
    return np.asarray(out, dtype=np.int32).reshape(-1, 2)


def make_edges(wl: Workload, seed: int = SEED):
    """(ii, jj) int32 arrays for a workload."""
    if wl.name == "C1":
        return np.array([0], np.int32), np.array([1], np.int32)
    pairs = ordered_pairs(wl.frames, wl.max_offset)
    rng = np.random.default_rng(seed)
    if wl.edges < len(pairs):
        idx = np.sort(rng.choice(len(pairs), size=wl.edges, replace=False))
        pairs = pairs[idx]
    return np.ascontiguousarray(pairs[:, 0]), np.ascontiguousarray(pairs[:, 1])


def grid_coords(h: int, w: int) -> np.ndarray:
    """Identity pixel grid [2, h, w] (ch0 = x, ch1 = y)."""
    ys, xs = np.meshgrid(np.arange(h, dtype=np.float32), np.arange(w, dtype=np.float32),
                         indexing="ij")
    return np.stack([xs, ys])


def make_coords_np(wl: Workload, M: int, seed: int = SEED + 1) -> np.ndarray:
    rng = np.random.default_rng(seed)
    g = grid_coords(wl.h, wl.w)[None]
    if wl.coord_noise == "uniform4":
        n = rng.uniform(-4.0, 4.0, size=(M, 2, wl.h, wl.w))
    else:
        n = rng.normal(0.0, wl.sigma, size=(M, 2, wl.h, wl.w))
    return (g + n).astype(np.float32)


def make_fmaps_np(wl: Workload, frames: int = None, seed: int = SEED + 2) -> np.ndarray:
    rng = np.random.default_rng(seed)
    K = wl.frames if frames is None else frames
    return rng.standard_normal((K, wl.channels, wl.h, wl.w), dtype=np.float32)


def make_device_inputs(wl: Workload, device, seed: int = SEED):
    """Feature maps and coordinates generated on the device (torch RNG, seeded)
    for the full-size benchmark workloads."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    ii, jj = make_edges(wl, seed)
    fm = torch.randn(wl.frames, wl.channels, wl.h, wl.w, generator=g, device=device)
    M = len(ii)
    base = torch.from_numpy(grid_coords(wl.h, wl.w)).to(device)[None]
    if wl.coord_noise == "uniform4":
        noise = torch.rand(M, 2, wl.h, wl.w, generator=g, device=device) * 8.0 - 4.0
    else:
        noise = torch.randn(M, 2, wl.h, wl.w, generator=g, device=device) * wl.sigma
    coords = (base + noise).contiguous()
    return fm, ii, jj, coords


def random_poses(n: int, rng, trans: float = 0.1, angle: float = 0.05) -> np.ndarray:
    """Seeded camera poses [n, 7] (t_x t_y t_z q_x q_y q_z q_w, unit q) near the
    identity, as a keyframe window of a SLAM run would have; float32."""
    t = rng.normal(0, trans, (n, 3))
    axis = rng.normal(0, 1, (n, 3))
    axis /= np.linalg.norm(axis, axis=1, keepdims=True)
    half = 0.5 * rng.normal(0, angle, (n, 1))
    q = np.concatenate([axis * np.sin(half), np.cos(half)], 1)
    return np.concatenate([t, q], 1).astype(np.float32)

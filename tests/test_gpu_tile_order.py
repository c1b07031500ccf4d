"""Window-row tile order of the fused kernel (dc_set_tile_order).

The order only changes which source pixels share a 128-pixel tile (a
pre-pass sorts each edge's pixels by the row of their level-0 window and the
source tile is gathered row by row), never a pixel's own arithmetic: every
output must equal the source-order output.  Checked at the frontend (C2) and
backend (C5) geometries and flows, at an odd geometry whose last tile is
partial, for every tensor-core precision, and for the automatic choice; a
sample of C5 edges is also compared with the oracle at the usual bars.
"""
import numpy as np
import pytest
import torch

from slam_hands_b200 import DroidCorrelation, configs

from test_gpu_parity import normwise
from test_gpu_workloads import _oracle_edges

pytestmark = pytest.mark.gpu


def _run(wl, fm, ii_d, jj_d, coords, precision, order, M):
    dc = DroidCorrelation(wl.h, wl.w, precision=precision, alpha=wl.alpha,
                          max_frames=wl.frames, max_edges=M)
    dc.set_frames(fm)
    dc.set_tile_order(order)
    out = dc.build_and_lookup(ii_d, jj_d, coords)
    assert dc.lib.dc_device_status(dc._ctx, None) == 0
    dc.close()
    return out


def _compare(a, b, what):
    same = torch.equal(a, b)
    err = (a - b).abs().max().item() / max(b.abs().max().item(), 1e-30)
    print(f"{what}: bit-identical {same}, max rel {err:.3e}")
    assert err < 1e-6, what


@pytest.mark.parametrize("name", ["C2", "C5"])
@pytest.mark.parametrize("precision", ["fp16", "bf16", "fp32x3"])
def test_window_row_order_matches_source_order(cuda, name, precision):
    wl = configs.WORKLOADS[name]
    fm, ii, jj, coords = configs.make_device_inputs(wl, cuda, seed=configs.SEED)
    M = min(len(ii), 256)
    ii_d = torch.from_numpy(ii[:M]).cuda()
    jj_d = torch.from_numpy(jj[:M]).cuda()
    co = coords[:M].contiguous()
    ref = _run(wl, fm, ii_d, jj_d, co, precision, "source", M)
    for order in ("window_row", "auto"):
        got = _run(wl, fm, ii_d, jj_d, co, precision, order, M)
        _compare(got, ref, f"{name} {precision} {order}")


def test_window_row_order_partial_tile_and_invalid_edges(cuda):
    # 41 x 73 = 2993 pixels: the last tile of every edge is partial; edge 2 has
    # an invalid slot and must give zeros in either order
    h, w, K, M = 41, 73, 4, 6
    g = torch.Generator(device=cuda).manual_seed(11)
    fm = torch.randn(K, 128, h, w, device=cuda, generator=g)
    ii = torch.tensor([0, 1, 99, 3, 2, 0], dtype=torch.int32, device=cuda)
    jj = torch.tensor([1, 2, 0, 0, 3, 3], dtype=torch.int32, device=cuda)
    ys, xs = torch.meshgrid(torch.arange(h, device=cuda), torch.arange(w, device=cuda),
                            indexing="ij")
    grid = torch.stack([xs, ys]).float()
    coords = (grid[None] + 8 * torch.randn(M, 2, h, w, device=cuda, generator=g)).contiguous()
    coords[4, :, 3, 5] = float("nan")
    outs = {}
    for order in ("source", "window_row"):
        dc = DroidCorrelation(h, w, precision="fp16", alpha=0.0625, max_frames=K, max_edges=M)
        dc.set_frames(fm)
        dc.set_tile_order(order)
        outs[order] = dc.build_and_lookup(ii, jj, coords)
        assert dc.lib.dc_device_status(dc._ctx, None) == 0
        dc.close()
    assert torch.equal(outs["window_row"][2], torch.zeros_like(outs["window_row"][2]))
    a, b = outs["window_row"], outs["source"]
    fin = torch.isfinite(b)
    assert torch.equal(torch.isfinite(a), fin)
    _compare(torch.where(fin, a, 0), torch.where(fin, b, 0), "41x73 window_row")


def test_window_row_order_c5_oracle(cuda, oracle):
    wl = configs.WORKLOADS["C5"]
    fm, ii, jj, coords = configs.make_device_inputs(wl, cuda, seed=configs.SEED)
    M = len(ii)
    ii_d = torch.from_numpy(ii).cuda()
    jj_d = torch.from_numpy(jj).cuda()
    out = _run(wl, fm, ii_d, jj_d, coords, "fp16", "window_row", M)
    rng = np.random.default_rng(configs.SEED + 9)
    idx = np.sort(rng.choice(M, 8, replace=False))
    frames = np.unique(np.concatenate([ii[idx], jj[idx]]))
    fm_host = np.zeros((wl.frames, wl.channels, wl.h, wl.w), np.float32)
    fm_host[frames] = fm[torch.from_numpy(frames).cuda()].cpu().numpy()
    got = out[torch.from_numpy(idx).cuda()].cpu().numpy()
    exp = _oracle_edges(oracle, fm_host, ii, jj, coords.cpu().numpy(), wl.alpha, "fp16", idx)
    err = normwise(got, exp)
    print(f"C5 window_row fp16: 8 of {M} edges normwise {err:.3e}")
    assert err < 1e-4


def test_tile_order_scratch_is_counted_once(cuda):
    h, w, M = 24, 32, 5
    dc = DroidCorrelation(h, w, precision="fp16", alpha=0.0625, max_frames=2, max_edges=M)
    before = dc.context_bytes
    dc.set_tile_order("auto")
    grown = dc.context_bytes
    assert grown - before == M * (3 * h * w + 1) * 4
    dc.set_tile_order("window_row")
    dc.set_tile_order("source")
    assert dc.context_bytes == grown  # the scratch is allocated once and kept
    with pytest.raises(Exception):
        dc.set_tile_order("rows")
    dc.close()

"""The correlation encoder's first layer (dc_corr_encode, dc_build_lookup_encode):
out = fp16(relu(W corr + b)), the reference's corr_enc_0 1x1 convolution 196 ->
128 + relu_inplace + round_to_fp16 (cuda_slam/main.cu:552-553, :603-606).

Bars: against the float64 oracle on the same fp16-rounded features and
weights, normwise <= 2e-3 (the output's own fp16 rounding plus fp32
accumulation order); against the oracle on the unrounded fp32 inputs and
against cuDNN's convolution (torch.nn.functional.conv2d, the reference's
library call on float tensors), normwise <= 2e-2 (the tensor-core precision
bar), max-abs error printed."""
import math

import numpy as np
import pytest
import torch

from slam_hands_b200 import DroidCorrelation, configs

from test_gpu_parity import normwise, oracle_alt


def _weights(seed, ci=196, co=128):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((co, ci)) / math.sqrt(ci)).astype(np.float32)
    b = (0.1 * rng.standard_normal(co)).astype(np.float32)
    return w, b


def test_oracle_encoder_matches_loops(oracle):
    rng = np.random.default_rng(3)
    corr = rng.standard_normal((2, 5, 3, 4)).astype(np.float32)
    w = rng.standard_normal((6, 5)).astype(np.float32)
    b = rng.standard_normal(6).astype(np.float32)
    got = oracle.corr_encode(corr, w, b)
    assert got.dtype == np.float16
    for m in range(2):
        for o in range(6):
            for y in range(3):
                for x in range(4):
                    v = sum(float(w[o, c]) * float(corr[m, c, y, x]) for c in range(5)) + float(b[o])
                    assert got[m, o, y, x] == np.float16(max(v, 0.0))


@pytest.mark.gpu
@pytest.mark.parametrize("h,w,M", [(48, 64, 3), (41, 73, 2), (5, 9, 1)])
def test_corr_encode_vs_oracle_and_cudnn(cuda, oracle, h, w, M):
    rng = np.random.default_rng(h * w)
    levels = 4 if min(h, w) >= 8 else 1
    ci = levels * 49
    corr = rng.standard_normal((M, ci, h, w)).astype(np.float32)
    W, b = _weights(h + w, ci=ci)
    dc = DroidCorrelation(h, w, levels=levels, max_frames=1)
    dc.set_corr_encoder(torch.from_numpy(W).cuda(), torch.from_numpy(b).cuda())
    out = dc.corr_encode(torch.from_numpy(corr).cuda())
    assert dc.lib.dc_device_status(dc._ctx, None) == 0
    got = out.float().cpu().numpy()
    r16 = lambda a: a.astype(np.float16).astype(np.float32)
    exp16 = oracle.corr_encode(r16(corr), r16(W), b).astype(np.float32)
    e1 = normwise(got, exp16)
    exp = oracle.corr_encode(corr, W, b).astype(np.float32)
    e2 = normwise(got, exp)
    ref = torch.relu(torch.nn.functional.conv2d(torch.from_numpy(corr).cuda(),
                                                torch.from_numpy(W).cuda()[:, :, None, None],
                                                torch.from_numpy(b).cuda()))
    ref = ref.half().float().cpu().numpy()
    e3 = normwise(got, ref)
    print(f"{h}x{w}: same-rounded {e1:.2e}, fp32 oracle {e2:.2e} (maxabs "
          f"{np.abs(got - exp).max():.2e}), cuDNN {e3:.2e}")
    assert e1 < 2e-3 and e2 < 2e-2 and e3 < 2e-2


@pytest.mark.gpu
@pytest.mark.parametrize("precision", ["fp16", "fp32"])
def test_build_lookup_encode_c2(cuda, oracle, precision):
    wl = configs.WORKLOADS["C2"]
    fm = configs.make_fmaps_np(wl)
    ii, jj = configs.make_edges(wl)
    ii, jj = ii[:8], jj[:8]
    coords = configs.make_coords_np(wl, len(ii))
    W, b = _weights(5)
    dc = DroidCorrelation(wl.h, wl.w, precision=precision, alpha=wl.alpha, max_frames=wl.frames)
    dc.set_frames(torch.from_numpy(fm).cuda())
    dc.set_corr_encoder(torch.from_numpy(W).cuda(), torch.from_numpy(b).cuda())
    out, corr = dc.build_lookup_encode(ii, jj, torch.from_numpy(coords).cuda())
    assert dc.lib.dc_device_status(dc._ctx, None) == 0
    # the intermediate is the fused lookup's output, the encoding is of it
    same = dc.build_and_lookup(ii, jj, torch.from_numpy(coords).cuda())
    assert torch.equal(corr, same)
    exp_corr = oracle_alt(oracle, fm, ii, jj, coords, wl.alpha, "fp32")
    exp = oracle.corr_encode(exp_corr, W, b).astype(np.float32)
    got = out.float().cpu().numpy()
    err = normwise(got, exp)
    print(f"C2 {precision}: encoded normwise {err:.2e} maxabs {np.abs(got - exp).max():.2e}")
    assert err < 2e-2


@pytest.mark.gpu
def test_encoder_errors(cuda):
    from slam_hands_b200 import DroidCorrError
    dc = DroidCorrelation(12, 16, max_frames=2)
    with pytest.raises(DroidCorrError):  # no weights yet
        dc.corr_encode(torch.zeros(1, 196, 12, 16, device="cuda"))
    with pytest.raises(ValueError):
        dc.set_corr_encoder(torch.zeros(64, 196, device="cuda"), torch.zeros(64, device="cuda"))

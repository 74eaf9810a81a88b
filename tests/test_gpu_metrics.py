"""Evaluation metrics on the GPU (aeisu_distortion through aeisu_b200.metrics) against the
reference's own scores (golden fixture) and the FP64 oracle.  Tolerance: 2e-10 absolute on
y_mse and y_ssim, the reference's own tolerance for these figures
(research/archival_sources/paper_bench/control_ablation_evaluate.py:82); the kernel's window
sums are separable, so they agree with the 2-D convolution to FP64 rounding, not bit for bit."""
import math

import numpy as np
import pytest

from oracle import metrics_np as M
from aeisu_b200 import metrics
from aeisu_b200.synthetic import make_frame
from test_metrics import golden_cases

pytestmark = pytest.mark.gpu
TOL = 2e-10


def close(got, want):
    assert got["y_mse"] == pytest.approx(want["y_mse"], rel=0, abs=TOL)
    assert got["y_ssim"] == pytest.approx(want["y_ssim"], rel=0, abs=TOL)
    if math.isinf(want["y_psnr"]):
        assert math.isinf(got["y_psnr"]) and got["y_mse"] == 0
    else:
        assert got["y_psnr"] == pytest.approx(want["y_psnr"], rel=1e-9)


def pair(seed, h, w, noise=0.03):
    t = make_frame(seed, h, w).astype(np.float32).transpose(2, 0, 1) / np.float32(255)
    p = t + np.random.default_rng(seed).normal(0, noise, t.shape).astype(np.float32)
    return np.ascontiguousarray(p), np.ascontiguousarray(t)


@pytest.mark.parametrize("case", range(6))
def test_golden_reference_scores(case):
    pred, target, crop, want = golden_cases()[case]
    got = metrics.distortion(pred, target, crop)
    close(got, {"y_mse": want[0], "y_psnr": want[1], "y_ssim": want[2]})


@pytest.mark.parametrize("h,w,crop", [
    (15, 15, 2),      # smallest frame for crop 2
    (40, 132, 2),     # window grid 118 wide: exactly one strip
    (40, 133, 2),     # 119: a second strip of one column
    (33, 246, 0),     # 236: two full strips
    (33, 247, 0),     # 237
    (300, 90, 7),     # several bands
    (11, 11, 0),      # a single window
    (257, 301, 3),
])
def test_matches_oracle(h, w, crop):
    p, t = pair(h * 1000 + w, h, w)
    close(metrics.distortion(p, t, crop), M.distortion(p, t, crop))


def test_large_frame_matches_oracle():
    p, t = pair(7, 720, 1280, 0.01)
    close(metrics.distortion(p, t), M.distortion(p, t))


def test_batch_device_and_host_agree():
    import torch
    ps, ts = zip(*(pair(900 + i, 70, 150) for i in range(4)))
    P, T = np.stack(ps), np.stack(ts)
    single = [metrics.distortion(P[i], T[i]) for i in range(4)]
    batch = metrics.distortion_batch(P, T)
    dev = metrics.distortion_batch(torch.from_numpy(P).cuda(), torch.from_numpy(T).cuda())
    assert batch == single          # the split of a frame does not depend on the batch
    assert dev == batch             # device and host inputs run the same kernel on the same values
    for i in range(4):
        close(batch[i], M.distortion(P[i], T[i]))


def test_identical_images():
    _, t = pair(31, 64, 64)   # in [0, 1], so the prediction's clamp leaves it as it is
    s = metrics.distortion(t, t.copy())
    assert s["y_mse"] == 0 and math.isinf(s["y_psnr"]) and s["y_ssim"] == pytest.approx(1.0, abs=1e-15)


def test_clamp_applies_to_the_prediction_only():
    p, t = pair(32, 48, 48, 0.3)   # many prediction values outside [0, 1]
    assert (p > 1).any() and (p < 0).any()
    close(metrics.distortion(p, t), M.distortion(p, t))
    # an out-of-range target is not clamped
    close(metrics.distortion(t, p), M.distortion(t, p))


@pytest.mark.parametrize("where", ["inside", "border", "target"])
def test_non_finite_values_raise(where):
    p, t = pair(33, 40, 40)
    if where == "inside":
        p[1, 20, 20] = np.nan
    elif where == "border":
        p[2, 0, 39] = np.inf   # cropped away, still checked as the reference checks whole images
    else:
        t[0, 39, 1] = -np.inf
    with pytest.raises(ValueError, match="finite"):
        metrics.distortion(p, t)
    P = np.stack([pair(34, 40, 40)[0], p])
    T = np.stack([pair(34, 40, 40)[1], t])
    with pytest.raises(ValueError, match="finite"):
        metrics.distortion_batch(P, T)

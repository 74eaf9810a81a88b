"""FP64 numpy restatement of the reference's evaluation metrics (TEST ORACLE ONLY).

Only tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
this module.  It follows aeisu/metrics.py:11-39 (paths relative to the AELabs42/AEISU
checkout): encoded BT.601 luma, Y MSE / PSNR and the Gaussian 11x11 (sigma 1.5) SSIM over
valid windows, all in FP64, the window applied as the full 2-D outer-product kernel as the
reference's ``F.conv2d`` applies it.
"""
from __future__ import annotations

import math

import numpy as np

LUMA_WEIGHTS = np.array([65.481, 128.553, 24.966], np.float64)   # metrics.py:12


def luma(rgb):
    """metrics.py:11-14: ((rgb * weights).sum(0) + 16) / 255 on FP64 CHW, keeps the channel axis."""
    rgb = np.asarray(rgb, np.float64)
    s = rgb[0] * LUMA_WEIGHTS[0] + rgb[1] * LUMA_WEIGHTS[1]
    s = s + rgb[2] * LUMA_WEIGHTS[2]
    return ((s + 16) / 255)[None]


def gaussian_window():
    """metrics.py:29-32: 11 taps at -5..5, sigma 1.5, normalised; window = outer product."""
    c = np.arange(11, dtype=np.float64) - 5
    g = np.exp(-(c * c) / (2 * 1.5 ** 2))
    g = g / g.sum()
    return g[:, None] * g[None, :]


def _smooth(img, window):
    """Valid 2-D correlation of an [H, W] FP64 image with the 11x11 window (F.conv2d, metrics.py:33-34)."""
    v = np.lib.stride_tricks.sliding_window_view(img, window.shape)
    return np.einsum("ijkl,kl->ij", v, window)


def distortion(prediction, target, crop=2):
    """metrics.py:17-39 on float CHW arrays; raises ValueError exactly where the reference does."""
    prediction = np.asarray(prediction)
    target = np.asarray(target)
    if prediction.shape != target.shape or prediction.ndim != 3:
        raise ValueError("Prediction and target must be same-size CHW RGB")
    if not np.isfinite(prediction).all() or not np.isfinite(target).all():
        raise ValueError("Prediction and target must be finite")
    if crop < 0 or min(prediction.shape[-2:]) < 11 + crop * 2:
        raise ValueError("Images are too small for the border crop and 11x11 SSIM window")
    a = np.clip(prediction, 0, 1).astype(np.float64)
    b = target.astype(np.float64)
    if crop:
        a, b = a[:, crop:-crop, crop:-crop], b[:, crop:-crop, crop:-crop]
    y1, y2 = luma(a)[0], luma(b)[0]
    mse = float(np.square(y1 - y2).mean())
    window = gaussian_window()
    mu1, mu2 = _smooth(y1, window), _smooth(y2, window)
    var1 = _smooth(y1 * y1, window) - mu1 * mu1
    var2 = _smooth(y2 * y2, window) - mu2 * mu2
    cov = _smooth(y1 * y2, window) - mu1 * mu2
    c1, c2 = .01 ** 2, .03 ** 2
    ssim = ((2 * mu1 * mu2 + c1) * (2 * cov + c2)) / ((mu1 * mu1 + mu2 * mu2 + c1) * (var1 + var2 + c2))
    return {"y_mse": mse, "y_psnr": math.inf if mse == 0 else -10 * math.log10(mse), "y_ssim": float(ssim.mean())}

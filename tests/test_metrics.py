"""Evaluation metrics, host side: the FP64 oracle (oracle/metrics_np.py) against the reference's
own distortion() outputs (tests/golden/metrics_distortion.npz, from make_metrics_golden.py), and
the argument checks of aeisu_b200.metrics / aeisu_distortion that run before any GPU work."""
import math

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import metrics_np as M
from aeisu_b200 import metrics


def golden_cases():
    d = np.load(GOLDEN / "metrics_distortion.npz")
    return [(d[f"pred{i}"], d[f"target{i}"], int(d[f"crop{i}"]), d[f"scores{i}"]) for i in range(int(d["cases"]))]


@pytest.mark.parametrize("case", range(6))
def test_oracle_matches_reference_scores(case):
    pred, target, crop, want = golden_cases()[case]
    s = M.distortion(pred, target, crop)
    assert s["y_mse"] == pytest.approx(want[0], rel=0, abs=1e-15)
    if math.isinf(want[1]):
        assert math.isinf(s["y_psnr"])
    else:
        assert s["y_psnr"] == pytest.approx(want[1], rel=1e-12)
    assert s["y_ssim"] == pytest.approx(want[2], rel=0, abs=1e-13)


def test_oracle_error_behaviour():
    a = np.zeros((3, 20, 20), np.float32)
    with pytest.raises(ValueError, match="same-size"):
        M.distortion(a, a[:, :19])
    b = a.copy()
    b[0, 0, 0] = np.nan
    with pytest.raises(ValueError, match="finite"):
        M.distortion(b, a)
    with pytest.raises(ValueError, match="too small"):
        M.distortion(a[:, :14], a[:, :14], crop=2)


def test_gaussian_window_is_normalised():
    w = M.gaussian_window()
    assert w.shape == (11, 11) and abs(w.sum() - 1) < 1e-15 and np.allclose(w, w.T)


def test_mirror_rejects_bad_arguments_before_gpu_work():
    a = np.zeros((3, 20, 20), np.float32)
    with pytest.raises(ValueError, match="same-size"):
        metrics.distortion(a, a[:, :19])
    with pytest.raises(ValueError, match="same-size"):
        metrics.distortion(a[:2], a[:2])
    with pytest.raises(TypeError):
        metrics.distortion(a.astype(np.float64), a)
    # size and crop are checked by the library before it touches a device
    with pytest.raises(ValueError, match="too small"):
        metrics.distortion(a[:, :14], a[:, :14], crop=2)
    with pytest.raises(ValueError, match="too small"):
        metrics.distortion(a, a, crop=-1)
    with pytest.raises(ValueError, match="same-size"):
        metrics.distortion_batch(a, a)

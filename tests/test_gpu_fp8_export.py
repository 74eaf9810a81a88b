"""FP8 exporter on the GPU: the FP32 route's calibration statistics against their CPU
restatement, and artifacts exported from the reference's folded checkpoints held to the mixed
route's bar (mean >= 50 dB, every frame >= 44 dB against the same checkpoint's FP32 route)."""
import numpy as np
import pytest

import spyr8_helpers as H
from conftest import staged
from oracle import aeisu_np as O
from aeisu_b200 import Model, load_model
from aeisu_b200._lib import AeisuError
from aeisu_b200 import fp8_export as X
from aeisu_b200.synthetic import make_frames

pytestmark = pytest.mark.gpu


def _psnr(ref_chw, got_chw):
    return O.psnr(np.clip(got_chw, 0, 1), np.clip(ref_chw, 0, 1))


def test_activation_stats_match_the_cpu_restatement():
    import torch
    state, l1 = X.load_folded_state(staged("aeisu_area.pt"))
    frames = make_frames(3100, 2, 72, 100)
    model = Model.from_folded_state(state, "cuda:0", "fp32", l1)
    try:
        peaks, means = model.activation_stats(frames)
        want_p, want_m = H.activation_stats(state, frames)
        np.testing.assert_allclose(peaks, want_p, rtol=2e-5)
        np.testing.assert_allclose(means, want_m, rtol=1e-4, atol=1e-6)
        p2, m2 = model.activation_stats(torch.from_numpy(frames).cuda())   # device input
        np.testing.assert_array_equal(p2, peaks)
        np.testing.assert_allclose(m2, means, rtol=1e-6, atol=1e-9)
    finally:
        model.close()
    fp16 = Model.from_folded_state(state, "cuda:0", "fp16", l1)
    try:
        with pytest.raises(AeisuError):
            fp16.activation_stats(frames)
    finally:
        fp16.close()


def _mixed_psnrs(data, ckpt):
    ref = load_model(staged(ckpt), "cuda:0", "fp32")
    mixed = Model.from_spyr8_bytes(data, "cuda:0", "mixed")
    try:
        ps = []
        for seed in range(2000, 2008):   # held out: not among the calibration frames
            src = O.u8_to_chw(make_frames(seed, 1, 128, 128)[0])
            ps.append(_psnr(ref.upscale_f32(src, 0), mixed.upscale_f32(src, 0)))
        return np.array(ps)
    finally:
        ref.close()
        mixed.close()


@pytest.mark.parametrize("ckpt", ["aeisu_area.pt", "aeisu_bicubic.pt"])
def test_exported_artifact_meets_the_mixed_bar(ckpt):
    calib = make_frames(3200, 8, 128, 128)
    data = X.export_spyr8(staged(ckpt), calib, "cuda:0")
    ps = _mixed_psnrs(data, ckpt)
    assert ps.mean() >= 50.0 and ps.min() >= 44.0, np.round(ps, 2).tolist()


def test_export_does_at_least_as_well_as_the_shipped_artifact():
    """Same checkpoint (aeisu_area.pt, from which adaptive_fp8.bin was exported) and frames."""
    calib = make_frames(3200, 8, 128, 128)
    ours = _mixed_psnrs(X.export_spyr8(staged("aeisu_area.pt"), calib, "cuda:0"), "aeisu_area.pt")
    shipped = _mixed_psnrs(staged("adaptive_fp8.bin").read_bytes(), "aeisu_area.pt")
    assert ours.mean() >= shipped.mean() - 0.5, (ours.mean(), shipped.mean())


def test_scale_search_never_loses():
    state, l1 = X.load_folded_state(staged("aeisu_area.pt"))
    calib = make_frames(3300, 3, 96, 96)
    peaks, means = X.calibrate(state, calib, "cuda:0", l1)
    scales = np.maximum(peaks, 1e-6) / 448
    best, before, after = X.search_scales(state, scales, means, calib, "cuda:0", l1, factors=(0.5, 2.0))
    assert after >= before
    assert best.shape == (10,) and np.all(best > 0)

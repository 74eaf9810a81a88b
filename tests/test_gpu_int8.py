"""INT8/FP16 route (shader_precision_v1 artifact) on the GPU against its CPU restatement
(oracle/mixed_np.py, mode "int8") and against the FP32 route of the checkpoint it was exported
from (aeisu_area.pt: the artifact's FP16 weights are that checkpoint's, rounded).

The reference runs this route only on an RTX 5090 (optimized/shader/runtime.py:14-17), so parity
is with the restatement of its quantisation points; the distance from FP32 is the bar the
reference sets for its reduced-precision routes (>= 35 dB, SrcPyrRuntimeTest.cpp:454-457),
here bounded tighter by what the restatement itself reaches on these scenes."""
import numpy as np
import pytest

from conftest import staged
from oracle import aeisu_np as O
from oracle import mixed_np as M
from aeisu_b200 import _lib, load_model
from aeisu_b200.synthetic import make_frame, make_frames

pytestmark = pytest.mark.gpu


def psnr_vs(ref_chw, got_chw):
    return O.psnr(np.clip(got_chw, 0, 1), np.clip(ref_chw, 0, 1))


@pytest.fixture(scope="module")
def int8_model():
    m = load_model(staged("aeisu_int8_fp16.pt"), "cuda:0")
    yield m
    m.close()


@pytest.fixture(scope="module")
def restated():
    import torch
    rec = torch.load(staged("aeisu_int8_fp16.pt"), map_location="cpu", weights_only=True)
    return M.QuantizedModel(M.int8_record_tensors(rec), "int8")


def test_route_report(int8_model):
    assert int8_model.precision == "int8" and "int8" in int8_model.report


@pytest.mark.parametrize("seed, h, w", [(801, 256, 256), (802, 96, 160), (803, 70, 130)])
def test_matches_restatement(int8_model, restated, seed, h, w):
    """Integer sums are exact on both sides; differences come only from f16/FP32 roundings
    whose accumulation order differs, flipping a few int8 codes."""
    src = O.u8_to_chw(make_frame(seed, h, w))
    p = psnr_vs(O.upscale(restated, src, 0), int8_model.upscale_f32(src, 0))
    assert p >= 60.0, f"{p:.2f} dB vs restatement"


def test_close_to_fp32_route(int8_model):
    ref = O.load_folded(staged("aeisu_area.pt"))
    ps = []
    for seed in range(2000, 2006):
        src = O.u8_to_chw(make_frame(seed, 128, 128))
        ps.append(psnr_vs(O.upscale(ref, src, 0), int8_model.upscale_f32(src, 0)))
    assert np.mean(ps) >= 44.0 and min(ps) >= 40.0, [round(p, 2) for p in ps]


def test_batch_tile_and_device_io(int8_model):
    import torch
    frames = make_frames(11, 3, 64, 96)
    batch = int8_model.upscale_u8(frames, 0)
    for i in range(3):
        np.testing.assert_array_equal(int8_model.upscale_u8(frames[i], 0), batch[i])
    dev = int8_model.upscale_u8(torch.from_numpy(frames).cuda(), 0).cpu().numpy()
    np.testing.assert_array_equal(dev, batch)
    tiled = int8_model.upscale_u8(frames, 32)
    assert O.psnr(tiled.astype(np.float64) / 255, batch.astype(np.float64) / 255) >= 40


def test_precision_rules():
    with pytest.raises(ValueError, match="only at precision int8"):
        load_model(staged("aeisu_int8_fp16.pt"), "cuda:0", "fp16")
    with pytest.raises(_lib.AeisuError, match="INT8 precision needs"):
        load_model(staged("aeisu_area.pt"), "cuda:0", "int8")

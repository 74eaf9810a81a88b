"""Reconstruction fused into the controller's last kernel (k_tc_refine_head) against the unfused
pair (k_tc_refine_tail, then k_tc_head over coefficients in device memory), on every tensor-core
route.  Both compute the same clamped f16 coefficients, the same filter weights on the tensor core
and the same accumulation order of the 5 x 5 x 3 apply, so their frames must agree bit for bit.
The unfused pair is itself checked against the CPU restatement and the reference's goldens by the
other GPU tests; this file pins the fused kernel to it on the shapes and I/O forms that exercise
its work decomposition (strips, bands, core rectangles of tiles and bands, two-stream batches)."""
import numpy as np
import pytest

from conftest import staged
from aeisu_b200 import load_model
from aeisu_b200.synthetic import make_frame, make_frames

pytestmark = pytest.mark.gpu


def both(model, fn):
    unfused = fn()   # the default
    model.set_fused_head(True)
    try:
        fused = fn()
    finally:
        model.set_fused_head(False)
    return unfused, fused


def as_np(x):
    return x.cpu().numpy() if hasattr(x, "cpu") else np.asarray(x)


@pytest.fixture(scope="module", params=["fp16", "mixed", "int8"])
def model(request):
    if request.param == "int8":
        m = load_model(staged("aeisu_int8_fp16.pt"), "cuda:0")
    else:
        m = load_model(staged("adaptive_fp8.bin"), "cuda:0", request.param)
    yield m
    m.close()


@pytest.mark.parametrize("h,w,tile", [(1, 1, 0), (5, 7, 0), (33, 65, 0), (72, 128, 0), (257, 300, 0),
                                      (150, 200, 64), (120, 512, 128), (97, 131, 96)])
def test_uint8_frames_equal(model, h, w, tile):
    frame = make_frame(900 + h + w, h, w)
    unfused, fused = both(model, lambda: model.upscale_u8(frame, tile))
    np.testing.assert_array_equal(fused, unfused)


def test_two_stream_batch_equal(model):
    # nine regions: the engine runs the batch as two halves on two streams
    frames = make_frames(910, 9, 64, 96)
    unfused, fused = both(model, lambda: model.upscale_u8(frames, 0))
    np.testing.assert_array_equal(fused, unfused)


def test_float_io_equal(model):
    # float32 CHW source and unclipped float32 destination (upscale_f32, forward)
    frames = make_frames(920, 2, 40, 72).astype(np.float32).transpose(0, 3, 1, 2) / 255.0
    frames[1, :, 3:9, 5:30] *= 1.7   # values above 1: the unclipped path keeps them
    for tile in (0, 32):
        unfused, fused = both(model, lambda: model.upscale_f32(frames, tile))
        np.testing.assert_array_equal(fused, unfused)
    unfused, fused = both(model, lambda: model(frames[:, :, :32, :64]))
    np.testing.assert_array_equal(fused, unfused)


def test_device_io_and_bands_equal(model):
    import torch
    frame = make_frame(930, 200, 300)
    dev = torch.from_numpy(frame).cuda()
    unfused, fused = both(model, lambda: as_np(model.upscale_u8(dev, 0)))
    np.testing.assert_array_equal(fused, unfused)
    for bands in (2, 3):
        for band in range(bands):
            unfused, fused = both(model, lambda: model.upscale_u8_band(frame, band, bands))
            np.testing.assert_array_equal(fused, unfused)


def test_nonfinite_source_is_reported(model):
    frames = np.full((1, 3, 24, 40), 0.5, np.float32)
    frames[0, 1, 7, 11] = np.nan
    try:
        for fused in (False, True):
            model.set_fused_head(fused)
            with pytest.raises(FloatingPointError):
                model.upscale_f32(frames, 0)
    finally:
        model.set_fused_head(False)


@pytest.mark.parametrize("h,w", [(720, 1280), (1080, 1920)])
def test_benchmarked_frame_sizes_equal(model, h, w):
    frame = make_frame(940 + h, h, w)
    unfused, fused = both(model, lambda: model.upscale_u8(frame, 0))
    np.testing.assert_array_equal(fused, unfused)

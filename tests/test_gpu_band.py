"""Row bands of a single frame (aeisu_upscale_u8_band): the split a huge frame takes across
GPUs, one band per GPU with recomputed 32-row halos (the tile halos of aeisu/runtime.py:89-99).
The union of the bands must equal the whole-frame upscale bit for bit on every route, because
the controller's receptive field is smaller than the halo."""
import numpy as np
import pytest

from conftest import staged
from aeisu_b200 import load_model
from aeisu_b200.synthetic import make_frame

pytestmark = pytest.mark.gpu

ROUTES = [("aeisu_area.pt", "fp32"), ("aeisu_area.pt", "fp16"), ("adaptive_fp8.bin", "mixed")]


@pytest.mark.parametrize("ckpt,precision", ROUTES)
@pytest.mark.parametrize("h,w", [(200, 300), (97, 131)])
def test_bands_reassemble_the_whole_frame(ckpt, precision, h, w):
    model = load_model(staged(ckpt), "cuda:0", precision)
    try:
        frame = make_frame(4100 + h, h, w)
        whole = model.upscale_u8(frame, 0)
        other = make_frame(4150 + h, h, w)
        for bands in (1, 2, 3, 8, 13):
            # a different frame first, so no output row of `frame` is left in the workspace
            model.upscale_u8(other, 0)
            out = np.zeros_like(whole)
            for b in range(bands):
                model.upscale_u8_band(frame, b, bands, out=out)
            np.testing.assert_array_equal(out, whole, err_msg=f"{bands} bands")
    finally:
        model.close()


def test_band_writes_only_its_rows_with_device_io():
    import torch
    model = load_model(staged("adaptive_fp8.bin"), "cuda:0", "mixed")
    try:
        frame = make_frame(4200, 160, 96)
        whole = model.upscale_u8(frame, 0)
        dev = torch.from_numpy(frame).cuda()
        bands = 4
        # padded height 192 = 6 groups of 32 rows -> bands of 64 padded rows; the fourth is empty
        seen = np.zeros(whole.shape[0], dtype=bool)
        for b in range(bands):
            out = torch.full(whole.shape, 7, dtype=torch.uint8, device="cuda")
            model.upscale_u8_band(dev, b, bands, out=out)
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            rows = np.nonzero((got != 7).any(axis=(1, 2)))[0]
            if b == 3:
                assert len(rows) == 0
                continue
            lo, hi = rows.min(), rows.max() + 1
            assert not seen[lo:hi].any(), "bands overlap"
            seen[lo:hi] = True
            np.testing.assert_array_equal(got[lo:hi], whole[lo:hi])
            assert (got[:lo] == 7).all() and (got[hi:] == 7).all()
        assert seen.all()
    finally:
        model.close()


def test_band_arguments_are_checked():
    model = load_model(staged("adaptive_fp8.bin"), "cuda:0", "mixed")
    try:
        frame = make_frame(4300, 64, 64)
        for band, bands in ((2, 2), (-1, 3), (0, 0)):
            with pytest.raises(ValueError):
                model.upscale_u8_band(frame, band, bands)
    finally:
        model.close()

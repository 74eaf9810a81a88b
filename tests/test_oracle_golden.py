"""Pin the numpy oracle against the reference's own outputs and known-answer tests.

Fixtures in tests/golden/ were produced by tests/golden/make_golden.py, which runs the
reference PyTorch implementation.  The KATs restate tests/test_reference.py:31-61, 109-117.
"""
import numpy as np
import pytest

from conftest import GOLDEN, staged
from oracle import aeisu_np as O
from aeisu_b200.synthetic import bilinear_base, random_folded_state


def test_folded_parameter_count():
    # tests/test_reference.py:69: 115,996 deployed parameters
    assert sum(int(np.prod(s)) for _, s in O.STATE_SHAPES) == 115996
    st = random_folded_state(0)
    assert set(st) == {k for k, _ in O.STATE_SHAPES}


def test_coefficient_clamp_kat():
    # tests/test_reference.py:31-34
    value = np.array([-20., -12., -4., -2., 0., 2., 4., 12., 20.], np.float32)
    expected = np.array([-2.5, -2.5, -2.1, -2., 0., 2., 2.1, 2.5, 2.5], np.float32)
    np.testing.assert_allclose(O.coefficient_clamp(value), expected, rtol=1.3e-6, atol=1e-5)
    d = np.load(GOLDEN / "reconstruction_kat.npz")
    np.testing.assert_array_equal(O.coefficient_clamp(d["clamp_in"]), d["clamp_out"])


def test_parity_packing_kat():
    # tests/test_reference.py:36-45: head channels are LR-parity-major
    meta = np.empty((1, 64, 2, 3), np.float32)
    for parity in range(4):
        for component in range(16):
            meta[:, parity * 16 + component] = parity * .1 + component * .001
    coeff = O.unpack_coefficients(meta)
    for y in range(4):
        for x in range(6):
            expected = np.arange(16) * .001 + (2 * (y % 2) + x % 2) * .1
            np.testing.assert_allclose(coeff[0, :, y, x], expected, rtol=1e-6, atol=1e-7)
    d = np.load(GOLDEN / "reconstruction_kat.npz")
    np.testing.assert_array_equal(O.unpack_coefficients(d["meta"]), d["unpacked"])


def test_basis_projection_contract():
    # tests/test_reference.py:47-54 plus the reference's own projection of a fixed raw bank
    raw = np.random.default_rng(17).normal(size=(16, 4, 25)).astype(np.float32)
    basis = O.project_basis(raw)
    np.testing.assert_allclose(basis.sum(0), 0, atol=5e-8)
    assert np.abs(basis).sum(0).max() <= .5000002
    np.testing.assert_array_equal(O.project_basis(np.zeros_like(raw)), np.zeros((25, 16, 4)))
    d = np.load(GOLDEN / "reconstruction_kat.npz")
    np.testing.assert_allclose(O.project_basis(d["basis_raw"]), d["basis"], atol=5e-8, rtol=0)


def test_head_zero_model_is_bilinear():
    # tests/test_reference.py:56-61: coefficients 0 + exact bilinear base == 2x bilinear
    d = np.load(GOLDEN / "bilinear_identity.npz")
    st = random_folded_state(21)
    st["metadata_head.weight"][:] = 0
    st["metadata_head.bias"][:] = 0
    st["base_kernel"] = bilinear_base()
    out = O.FoldedModel(st)(d["source"])
    np.testing.assert_allclose(out, d["forward"], atol=3e-7, rtol=0)
    np.testing.assert_allclose(out, d["bilinear"], atol=3e-7, rtol=0)


@pytest.mark.parametrize("name", ["random_w11_f100_36x44", "random_w12_f101_69x83", "random_w13_f102_64x48"])
def test_random_weight_fixtures(name):
    d = np.load(GOLDEN / f"{name}.npz")
    model = O.FoldedModel(random_folded_state(int(d["weight_seed"])))
    src = O.u8_to_chw(d["frame"])
    h, w = src.shape[1:]
    py, px, ph, pw = O.pad_geometry(h, w)
    image = np.pad(src[None], ((0, 0), (0, 0), (py, ph - h - py), (px, pw - w - px)), mode="edge")
    meta = model.predict_coefficients(image)
    np.testing.assert_allclose(meta, d["meta"], atol=2e-5, rtol=2e-6)
    for tile in (0, 32):
        out = O.upscale(model, src, tile)
        np.testing.assert_allclose(out, d[f"upscale_tile{tile}"], atol=2e-6, rtol=0)


def test_tiled_equals_whole():
    # tests/test_reference.py:109-117 on the oracle itself
    model = O.FoldedModel(random_folded_state(3))
    src = np.random.default_rng(4).random((3, 69, 83), dtype=np.float32)
    whole, tiled = O.upscale(model, src, 0), O.upscale(model, src, 32)
    assert tiled.shape == (3, 138, 166)
    np.testing.assert_allclose(tiled, whole, atol=2e-6, rtol=2e-6)


def test_upscale_argument_errors():
    model = O.FoldedModel(random_folded_state(3))
    with pytest.raises(ValueError):
        O.upscale(model, np.zeros((4, 8, 8), np.float32))
    with pytest.raises(ValueError):
        O.upscale(model, np.zeros((3, 8, 8), np.float32), tile=48)
    bad = np.zeros((3, 8, 8), np.float32)
    bad[0, 3, 3] = np.nan
    with pytest.raises(FloatingPointError):
        O.upscale(model, bad, 0)


@pytest.mark.parametrize("name", ["aeisu_area_f200_48x64_t0", "aeisu_area_f0_256x256_t0",
                                  "aeisu_bicubic_f300_150x200_t64"])
def test_trained_checkpoint_fixtures(name):
    d = np.load(GOLDEN / f"{name}.npz")
    path = staged(str(d["checkpoint"]))
    import hashlib
    assert hashlib.sha256(path.read_bytes()).hexdigest() == str(d["checkpoint_sha256"])
    model = O.load_folded(path)
    out = O.upscale(model, O.u8_to_chw(d["frame"]), int(d["tile"]))
    if "upscale_f32" in d:
        np.testing.assert_allclose(out, d["upscale_f32"], atol=2e-6, rtol=0)
    else:
        y, x = d["window_origin"]
        np.testing.assert_allclose(out[:, y:y + 128, x:x + 128], d["window_f32"], atol=2e-6, rtol=0)
    u8 = O.chw_to_u8(out)
    diff = np.abs(u8.astype(int) - d["upscale_u8"].astype(int))
    assert diff.max() <= 1 and (diff > 0).mean() <= 1e-4


def test_tile256_seams_at_full_size():
    """Config 4 of the benchmark set at its own size: aeisu_bicubic.pt on a 1920x1080 bicubic
    frame through the reference's tiled path (tile 256, 32-LR halos, aeisu/runtime.py:89-99).
    The oracle must reproduce the reference's float output on every row and column beside a tile
    seam and its uint8 output row by row."""
    import hashlib
    from aeisu_b200.synthetic import make_frame
    d = np.load(GOLDEN / "aeisu_bicubic_f400_1080x1920_t256.npz")
    path = staged(str(d["checkpoint"]))
    assert hashlib.sha256(path.read_bytes()).hexdigest() == str(d["checkpoint_sha256"])
    h, w, tile = int(d["h"]), int(d["w"]), int(d["tile"])
    frame = make_frame(int(d["seed"]), h, w, str(d["degradation"]))
    assert hashlib.sha256(frame.tobytes()).hexdigest() == str(d["frame_sha256"])
    out = O.upscale(O.load_folded(path), O.u8_to_chw(frame), tile)
    assert len(d["seam_rows"]) == 4 and len(d["seam_cols"]) == 7
    np.testing.assert_allclose(out[:, d["row_index"], :], d["rows_f32"], atol=2e-6, rtol=0)
    np.testing.assert_allclose(out[:, :, d["col_index"]], d["cols_f32"], atol=2e-6, rtol=0)
    sums = O.chw_to_u8(out).astype(np.int64).sum(axis=(1, 2))
    assert np.abs(sums - d["u8_row_sums"]).max() <= 4

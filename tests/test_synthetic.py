"""Seeded workload generators: determinism, value ranges, degradation arithmetic."""
import numpy as np

from aeisu_b200 import synthetic as S


def test_frames_are_deterministic_and_distinct():
    a = S.make_frame(7, 40, 56)
    b = S.make_frame(7, 40, 56)
    c = S.make_frame(8, 40, 56)
    assert a.dtype == np.uint8 and a.shape == (40, 56, 3)
    np.testing.assert_array_equal(a, b)
    assert np.abs(a.astype(int) - c).mean() > 5


def test_area_downsample_rounds_half_up():
    hr = np.array([[[0], [1]], [[1], [0]]], np.uint8)           # sum 2 -> (2+2)//4 = 1
    assert S.area_downsample(hr)[0, 0, 0] == 1
    hr = np.array([[[255], [254]], [[255], [255]]], np.uint8)   # sum 1019 -> 255
    assert S.area_downsample(hr)[0, 0, 0] == 255
    hr = np.random.default_rng(0).integers(0, 256, (8, 10, 3), dtype=np.uint8)
    ref = (hr.reshape(4, 2, 5, 2, 3).astype(int).sum((1, 3)) + 2) // 4
    np.testing.assert_array_equal(S.area_downsample(hr), ref)


def test_bicubic_downsample_preserves_constants():
    hr = np.full((16, 12, 3), 77, np.uint8)
    lr = S.bicubic_downsample(hr)
    assert lr.shape == (8, 6, 3)
    assert (lr == 77).all()


def test_scene_statistics():
    img = S.procedural_scene(128, 192, np.random.default_rng(3))
    assert img.dtype == np.float32 and img.min() >= 0 and img.max() <= 1
    assert img.std() > 0.05  # not flat: polygons, waves and lines


def test_random_state_is_seeded():
    a, b = S.random_folded_state(5), S.random_folded_state(5)
    for k in a:
        np.testing.assert_array_equal(a[k], b[k])

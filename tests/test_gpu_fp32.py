"""FP32 route on the GPU, through the C ABI, against the CPU oracle and the reference's
golden outputs.  Bar (north star): max abs <= 1e-4 before quantisation; after uint8
rounding at most +-1 LSB on at most 0.1% of values."""
import numpy as np
import pytest

from conftest import GOLDEN, staged
from oracle import aeisu_np as O
from aeisu_b200 import Model, load_model, spyr8, upscale
from aeisu_b200.synthetic import make_frame, make_frames, random_folded_state

pytestmark = pytest.mark.gpu
ATOL = 1e-4


def assert_u8_close(got, ref):
    diff = np.abs(got.astype(int) - ref.astype(int))
    assert diff.max() <= 1, f"max LSB diff {diff.max()}"
    assert (diff > 0).mean() <= 1e-3, f"{(diff > 0).mean():.5f} of values differ by 1 LSB"


@pytest.fixture(scope="module")
def models():
    cache = {}

    def get(seed):
        if seed not in cache:
            cache[seed] = Model.from_folded_state(random_folded_state(seed), "cuda:0", "fp32")
        return cache[seed]
    yield get
    for m in cache.values():
        m.close()


@pytest.mark.parametrize("name", ["random_w11_f100_36x44", "random_w12_f101_69x83", "random_w13_f102_64x48"])
def test_golden_upscale_and_coefficients(models, name):
    d = np.load(GOLDEN / f"{name}.npz")
    model = models(int(d["weight_seed"]))
    src = O.u8_to_chw(d["frame"])
    for tile in (0, 32):
        got = upscale(model, src, tile)
        np.testing.assert_allclose(got, d[f"upscale_tile{tile}"], atol=ATOL, rtol=0)
    h, w = src.shape[1:]
    py, px, ph, pw = O.pad_geometry(h, w)
    image = np.pad(src[None], ((0, 0), (0, 0), (py, ph - h - py), (px, pw - w - px)), mode="edge")
    meta = model.predict_coefficients(image)
    np.testing.assert_allclose(meta, d["meta"], atol=ATOL, rtol=1e-5)


@pytest.mark.parametrize("h,w,tile", [(1, 1, 0), (5, 7, 0), (33, 65, 0), (33, 65, 32), (96, 64, 64),
                                      (130, 70, 96)])
def test_edge_sizes_against_oracle(models, h, w, tile):
    model = models(12)
    frame = make_frame(h * 1000 + w, h, w)
    ref = O.upscale(O.FoldedModel(random_folded_state(12)), O.u8_to_chw(frame), tile)
    got = upscale(model, O.u8_to_chw(frame), tile)
    assert got.shape == (3, 2 * h, 2 * w)
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=0)
    assert_u8_close(model.upscale_u8(frame, tile), O.chw_to_u8(ref))


def test_forward_on_padded_batch(models):
    model = models(13)
    x = np.random.default_rng(1).random((2, 3, 40, 48), dtype=np.float32)
    ref = O.FoldedModel(random_folded_state(13))(x)
    np.testing.assert_allclose(model(x), ref, atol=ATOL, rtol=0)


def test_batch_matches_single_frames(models):
    model = models(11)
    frames = make_frames(40, 3, 50, 62)
    batch = model.upscale_u8(frames, 0)
    for i in range(3):
        np.testing.assert_array_equal(batch[i], model.upscale_u8(frames[i], 0))
    tiled = model.upscale_u8(frames, 32)
    assert_u8_close(tiled, batch)


def test_device_io_matches_host_io(models):
    import torch
    model = models(11)
    frames = make_frames(50, 2, 48, 80)
    host = model.upscale_u8(frames, 0)
    dev = model.upscale_u8(torch.from_numpy(frames).cuda(), 0)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dev.cpu().numpy(), host)


def test_error_semantics(models):
    model = models(11)
    with pytest.raises(ValueError):
        upscale(model, np.zeros((3, 16, 16), np.float32), tile=48)
    with pytest.raises(ValueError):
        upscale(model, np.zeros((4, 16, 16), np.float32))
    bad = np.random.default_rng(0).random((3, 20, 20), dtype=np.float32)
    bad[1, 10, 10] = np.nan
    with pytest.raises(FloatingPointError):
        upscale(model, bad, 0)


def test_nonfinite_flag_resets(models):
    model = models(11)
    bad = np.full((3, 20, 20), np.inf, np.float32)
    with pytest.raises(FloatingPointError):
        upscale(model, bad, 0)
    out = model.upscale_u8(make_frame(3, 24, 24), 0)
    assert out.shape == (48, 48, 3)


def test_bounded_wait_times_out_and_recovers(models):
    model = models(12)
    frames = make_frames(0, 2, 720, 1280)
    model.set_timeout(1e-3)
    with pytest.raises(TimeoutError):
        model.upscale_u8(frames, 0)
    model.synchronize(timeout_ms=60000)
    model.set_timeout(60000)
    out = model.upscale_u8(frames[:1], 0)
    assert out.shape == (1, 1440, 2560, 3)


@pytest.mark.parametrize("name", ["aeisu_area_f200_48x64_t0", "aeisu_area_f0_256x256_t0",
                                  "aeisu_bicubic_f300_150x200_t64"])
def test_trained_checkpoints_against_reference_outputs(name):
    d = np.load(GOLDEN / f"{name}.npz")
    model = load_model(staged(str(d["checkpoint"])), "cuda:0", "fp32")
    try:
        tile = int(d["tile"])
        out = upscale(model, O.u8_to_chw(d["frame"]), tile)
        if "upscale_f32" in d:
            np.testing.assert_allclose(out, d["upscale_f32"], atol=ATOL, rtol=0)
        else:
            y, x = d["window_origin"]
            np.testing.assert_allclose(out[:, y:y + 128, x:x + 128], d["window_f32"], atol=ATOL, rtol=0)
        assert_u8_close(model.upscale_u8(d["frame"], tile), d["upscale_u8"])
    finally:
        model.close()


def test_spyr8_artifact_fp32_route():
    data = staged("adaptive_fp8.bin").read_bytes()
    state, basis = spyr8.folded_state_from_spyr8(spyr8.read_spyr8(data))
    oracle = O.FoldedModel(state, basis=basis)
    model = Model.from_spyr8_bytes(data, "cuda:0", "fp32")
    try:
        frame = make_frame(9, 72, 100)
        ref = O.upscale(oracle, O.u8_to_chw(frame), 0)
        np.testing.assert_allclose(upscale(model, O.u8_to_chw(frame), 0), ref, atol=ATOL, rtol=0)
    finally:
        model.close()


def test_full_1080p_frame_against_oracle():
    path = staged("aeisu_area.pt")
    frame = make_frame(1000, 1080, 1920)
    ref = O.upscale(O.load_folded(path), O.u8_to_chw(frame), 0)
    model = load_model(path, "cuda:0", "fp32")
    try:
        got = upscale(model, O.u8_to_chw(frame), 0)
        assert float(np.abs(got - ref).max()) <= ATOL
        assert_u8_close(model.upscale_u8(frame, 0), O.chw_to_u8(ref))
    finally:
        model.close()


def test_training_checkpoint_loads_folded(tmp_path):
    """load_model of a train.py-style checkpoint (training coordinates not folded) folds it as the
    reference's load_model does (aeisu/runtime.py:49-52) and matches the reference's upscale of
    it (tests/golden/training_checkpoint.npz) within the FP32 bar."""
    import torch
    from aeisu_b200.synthetic import seeded_training_state
    d = np.load(GOLDEN / "training_checkpoint.npz")
    state = seeded_training_state(random_folded_state(int(d["weight_seed"])), int(d["branch_seed"]),
                                  float(d["branch_std"]))
    path = tmp_path / "training.pt"
    torch.save({"model": {k: torch.from_numpy(v) for k, v in state.items()}, "basis_l1_scale": 0.5}, path)
    model = load_model(path, "cuda:0")
    try:
        got = upscale(model, O.u8_to_chw(d["frame"]), 0)
        np.testing.assert_allclose(got, d["upscale_f32"], atol=ATOL, rtol=0)
        assert_u8_close(model.upscale_u8(d["frame"], 0), O.chw_to_u8(d["upscale_f32"]))
    finally:
        model.close()

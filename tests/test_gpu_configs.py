"""Parity at the size of every benchmarked configuration (the workloads bench.py times):

* config 3: the mixed FP8/FP16 route on a 64-frame batch of 1280x720 frames;
* config 4: aeisu_bicubic.pt on 1920x1080 bicubic frames, tiled with tile 256, against the
  reference's own tiled output (tests/golden/aeisu_bicubic_f400_1080x1920_t256.npz);
* config 5: a 3840x2160 mixed frame, and one 7680x4320 input frame split into 8 row bands.

The FP32 side of each comparison is the numpy oracle, pinned to the reference by the golden
fixtures (tests/test_oracle_golden.py); the mixed route is also held to its CPU restatement
(oracle/mixed_np.py) at the artifact's own activation scales.  The north-star bars: FP32 within
1e-4, uint8 within 1 LSB on at most 0.1% of pixels, FP16 and mixed at least 50 dB against FP32."""
import hashlib
import multiprocessing as mp
import os

import numpy as np
import pytest

from conftest import GOLDEN, staged
from oracle import aeisu_np as O
from oracle import mixed_np as M
from aeisu_b200 import load_model, spyr8
from aeisu_b200.synthetic import make_frame

pytestmark = pytest.mark.gpu
MIN_PSNR = 50.0


def frames_in_pool(args):
    """Seeded frames rendered in a spawn pool (a fresh interpreter per worker, safe beside CUDA)."""
    procs = max(1, min(len(args), (os.cpu_count() or 2) - 1, 32))
    if procs == 1:
        return [make_frame(*a) for a in args]
    with mp.get_context("spawn").Pool(procs) as pool:
        return pool.starmap(make_frame, args)


def psnr(ref, got):
    return O.psnr(np.clip(got, 0, 1), np.clip(ref, 0, 1))


def u8_within_one_lsb(got, ref):
    diff = np.abs(got.astype(int) - ref.astype(int))
    return diff.max() <= 1 and (diff > 0).mean() <= 1e-3


@pytest.fixture(scope="module")
def mixed_artifact():
    data = staged("adaptive_fp8.bin").read_bytes()
    return data, M.QuantizedModel(spyr8.read_spyr8(data), "mixed"), O.load_folded(staged("aeisu_area.pt"))


def test_config3_mixed_720p_batch_of_64(mixed_artifact):
    """Four frames of one 64-frame 1280x720 batch (first, two inner, last): each equals the
    single-frame call bit for bit, follows the restatement, and is compared with FP32."""
    data, restated, fp32 = mixed_artifact
    frames = np.stack(frames_in_pool([(3000 + i, 720, 1280, "area") for i in range(64)]))
    model = load_model(staged("adaptive_fp8.bin"), "cuda:0", "mixed")
    try:
        batch = model.upscale_u8(frames, 0)
        assert batch.shape == (64, 1440, 2560, 3)
        lows = []
        for i in (0, 21, 42, 63):
            np.testing.assert_array_equal(batch[i], model.upscale_u8(frames[i], 0))
            src = O.u8_to_chw(frames[i])
            got = model.upscale_f32(src, 0)
            p = psnr(O.upscale(restated, src, 0), got)
            assert p >= 62.0, f"frame {i}: {p:.2f} dB against the restatement"
            lows.append(psnr(O.upscale(fp32, src, 0), got))
        print(f"config 3, mixed against FP32, frames 0/21/42/63: {[round(float(p), 2) for p in lows]} dB")
        assert min(lows) >= MIN_PSNR, [round(float(p), 2) for p in lows]
    finally:
        model.close()


@pytest.fixture(scope="module")
def tile256():
    d = np.load(GOLDEN / "aeisu_bicubic_f400_1080x1920_t256.npz")
    path = staged(str(d["checkpoint"]))
    assert hashlib.sha256(path.read_bytes()).hexdigest() == str(d["checkpoint_sha256"])
    frame = make_frame(int(d["seed"]), int(d["h"]), int(d["w"]), str(d["degradation"]))
    assert hashlib.sha256(frame.tobytes()).hexdigest() == str(d["frame_sha256"])
    ref = O.upscale(O.load_folded(path), O.u8_to_chw(frame), int(d["tile"]))
    return d, path, frame, ref


def test_config4_fp32_tile256_against_the_reference(tile256):
    d, path, frame, ref = tile256
    model = load_model(path, "cuda:0", "fp32")
    try:
        got = model.upscale_f32(O.u8_to_chw(frame), int(d["tile"]))
        # against the reference's own tiled output beside every seam, then the whole frame
        assert float(np.abs(np.clip(got[:, d["row_index"], :], 0, 1) - d["rows_f32"]).max()) <= 1e-4
        assert float(np.abs(np.clip(got[:, :, d["col_index"]], 0, 1) - d["cols_f32"]).max()) <= 1e-4
        assert float(np.abs(np.clip(got, 0, 1) - ref).max()) <= 1e-4
        u8 = model.upscale_u8(frame, int(d["tile"]))
        assert u8_within_one_lsb(u8, O.chw_to_u8(ref))
        assert np.abs(u8.astype(np.int64).sum(axis=(1, 2)) - d["u8_row_sums"]).max() <= 8
    finally:
        model.close()


def test_config4_fp16_tile256_seams(tile256):
    """The FP16 route at tile 256: 50 dB over the frame, and every row and column beside a seam
    held on its own, so that a wrong halo cannot hide in the frame-wide figure.  A batch of two
    frames gives each frame exactly its single-frame result."""
    d, path, frame, ref = tile256
    tile = int(d["tile"])
    model = load_model(path, "cuda:0", "fp16")
    try:
        got = np.clip(model.upscale_f32(O.u8_to_chw(frame), tile), 0, 1)
        p = psnr(ref, got)
        assert p >= MIN_PSNR, f"fp16 tile 256: {p:.2f} dB"
        body = float(np.abs(got - ref).max())
        rows = np.abs(got[:, d["row_index"], :] - d["rows_f32"]).max(axis=(0, 2))
        cols = np.abs(got[:, :, d["col_index"]] - d["cols_f32"]).max(axis=(0, 1))
        print(f"config 4 fp16: {p:.2f} dB, max error {body:.4f}, at seams rows {rows.max():.4f} cols {cols.max():.4f}")
        assert rows.max() <= max(body, 1e-3) and cols.max() <= max(body, 1e-3)
        seam_psnr = psnr(d["rows_f32"], got[:, d["row_index"], :]), psnr(d["cols_f32"], got[:, :, d["col_index"]])
        assert min(seam_psnr) >= MIN_PSNR, seam_psnr
        pair = np.stack([frame, make_frame(int(d["seed"]) + 1, int(d["h"]), int(d["w"]), str(d["degradation"]))])
        both = model.upscale_u8(pair, tile)
        np.testing.assert_array_equal(both[0], model.upscale_u8(frame, tile))
    finally:
        model.close()


@pytest.fixture(scope="module")
def frame4k():
    return make_frame(5000, 2160, 3840)


def test_config5_mixed_4k_frame(mixed_artifact, frame4k):
    data, restated, fp32 = mixed_artifact
    model = load_model(staged("adaptive_fp8.bin"), "cuda:0", "mixed")
    try:
        src = O.u8_to_chw(frame4k)
        got = model.upscale_f32(src, 0)
        assert got.shape == (3, 4320, 7680)
        p = psnr(O.upscale(restated, src, 0), got)
        assert p >= 62.0, f"4K: {p:.2f} dB against the restatement"
        u8 = model.upscale_u8(frame4k, 0)
        assert u8_within_one_lsb(u8, O.chw_to_u8(np.clip(got, 0, 1)))
        q = psnr(O.upscale(fp32, src, 0), got)
        print(f"config 5, 4K mixed against FP32: {q:.2f} dB")
        assert q >= MIN_PSNR, f"4K mixed against FP32: {q:.2f} dB"
    finally:
        model.close()


@pytest.mark.parametrize("precision", ["mixed", "fp16"])
def test_config5_8k_frame_in_8_bands(frame4k, precision):
    """One 7680x4320 input frame (the 4K scene mirrored 2x2) in 8 row bands, one call per band as
    the 8 GPUs of a box run them: the union equals the whole-frame call bit for bit."""
    import torch
    big = np.concatenate([np.concatenate([frame4k, frame4k[:, ::-1]], 1),
                          np.concatenate([frame4k[::-1], frame4k[::-1, ::-1]], 1)], 0)
    big = np.ascontiguousarray(big)
    assert big.shape == (4320, 7680, 3)
    model = load_model(staged("adaptive_fp8.bin"), "cuda:0", precision)
    try:
        src = torch.from_numpy(big).cuda()
        whole = model.upscale_u8(src, 0)
        bands = torch.zeros_like(whole)
        for b in range(8):
            model.upscale_u8_band(src, b, 8, out=bands)
        torch.cuda.synchronize()
        assert torch.equal(bands, whole)
    finally:
        model.close()

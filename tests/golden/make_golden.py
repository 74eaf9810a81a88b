"""Generate the golden parity fixtures from the reference PyTorch implementation.

Run where a checkout of the reference is available (its path via ``--reference``, or the
``AEISU_REFERENCE`` environment variable):

    python tests/golden/make_golden.py [--reference PATH]

It imports the reference's own ``aeisu`` package and records, for seeded synthetic
frames, the outputs of its public operator API (``aeisu.runtime.upscale``,
``FoldedAEISU.predict_coefficients``, ``FoldedAEISU.forward``) and of the
reconstruction helpers whose known-answer tests live in tests/test_reference.py.
The fixtures are committed; tests never need the reference at run time.

Weights: ``random_folded_state(seed)`` from ``aeisu_b200.synthetic`` (regenerated
bit-identically by the tests from the same seed), plus the reference's trained
``weights/aeisu_area.pt`` and ``weights/aeisu_bicubic.pt`` whose SHA-256 is stored
beside each output so a test can confirm it runs the same checkpoint.
"""
from __future__ import annotations

import argparse
import os
import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from aeisu_b200.synthetic import make_frame, random_folded_state  # noqa: E402


def sha256(path):
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


SECTIONS = ("kat", "random", "bilinear", "trained", "training", "tile256")
# config 4 of the benchmark set: aeisu_bicubic.pt, 1920x1080, tile 256, bicubic degradation
TILE256 = dict(checkpoint="aeisu_bicubic.pt", seed=400, h=1080, w=1920, tile=256, degradation="bicubic")
# the training checkpoint case: seeded training coordinates around random folded weights
TRAINING = dict(weight_seed=14, branch_seed=31, branch_std=0.01, frame_seed=210, h=48, w=64)


def seam_rows_cols(h, w, tile):
    """Output rows and columns where the reference's tiles meet (aeisu/runtime.py:81-99): the
    tile starts on the padded grid, in output coordinates of the cropped frame."""
    ey, ex = -h % 32, -w % 32
    py, px = 16 + ey // 2, 16 + ex // 2
    ph, pw = h + 32 + ey, w + 32 + ex
    rows = [2 * (y - py) for y in range(tile, ph, tile) if 0 < 2 * (y - py) < 2 * h]
    cols = [2 * (x - px) for x in range(tile, pw, tile) if 0 < 2 * (x - px) < 2 * w]
    return rows, cols


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AEISU_REFERENCE"),
                    help="checkout of the reference (default: $AEISU_REFERENCE)")
    ap.add_argument("--only", nargs="*", default=None, choices=SECTIONS,
                    help="write only these fixture groups (default: all)")
    args = ap.parse_args()
    want = lambda name: args.only is None or name in args.only
    if not args.reference:
        ap.error("give the reference checkout with --reference or AEISU_REFERENCE")
    sys.path.insert(0, args.reference)
    import torch
    from torch.nn import functional as F
    from aeisu.model import FoldedAEISU
    from aeisu.reconstruction import coefficient_clamp, project_basis, unpack_coefficients
    from aeisu.runtime import load_model, upscale

    torch.set_num_threads(4)

    def folded_from_state(state):
        model = FoldedAEISU()
        model.load_state_dict({k: torch.from_numpy(v) for k, v in state.items()}, strict=True)
        return model.eval().requires_grad_(False)

    def frame_chw(frame):
        return torch.from_numpy(frame).permute(2, 0, 1).float().div(255)

    def padded(src):
        h, w = src.shape[-2:]
        ey, ex = -h % 32, -w % 32
        py, px = 16 + ey // 2, 16 + ex // 2
        return F.pad(src[None], (px, 32 + ex - px, py, 32 + ey - py), mode="replicate")

    # 1. reconstruction known-answer tests (tests/test_reference.py:31-54)
    if want("kat"):
        kat(HERE, torch, coefficient_clamp, project_basis, unpack_coefficients)
    if want("random"):
        random_cases(torch, folded_from_state, frame_chw, padded, upscale)
    if want("bilinear"):
        bilinear(torch, F, folded_from_state)
    if want("trained"):
        trained(torch, Path(args.reference), load_model, upscale, frame_chw)
    if want("training"):
        training(torch, load_model, upscale, frame_chw)
    if want("tile256"):
        tile256(torch, Path(args.reference), load_model, upscale, frame_chw)
    print("golden fixtures written to", HERE)


def kat(HERE, torch, coefficient_clamp, project_basis, unpack_coefficients):
    clamp_in = np.array([-20., -12., -4., -2., 0., 2., 4., 12., 20.], np.float32)
    rng = np.random.default_rng(5)
    meta_small = rng.normal(0, 1.5, (2, 64, 3, 5)).astype(np.float32)
    raw = rng.normal(0, 0.3, (16, 4, 25)).astype(np.float32)
    np.savez_compressed(
        HERE / "reconstruction_kat.npz",
        clamp_in=clamp_in,
        clamp_out=coefficient_clamp(torch.from_numpy(clamp_in)).numpy(),
        meta=meta_small,
        unpacked=unpack_coefficients(torch.from_numpy(meta_small)).numpy(),
        basis_raw=raw,
        basis=project_basis(torch.from_numpy(raw)).numpy(),
    )



def random_cases(torch, folded_from_state, frame_chw, padded, upscale):
    """Random-weight models on seeded frames: full frame, tiled, coefficients."""
    cases = [(11, 100, 36, 44), (12, 101, 69, 83), (13, 102, 64, 48)]
    for wseed, fseed, h, w in cases:
        state = random_folded_state(wseed)
        model = folded_from_state(state)
        frame = make_frame(fseed, h, w)
        src = frame_chw(frame)
        with torch.inference_mode():
            image = padded(src)
            meta = model.predict_coefficients(image)
            forward = model(image)
            whole = upscale(model, src, 0)
            tiled = upscale(model, src, 32)
        np.savez_compressed(
            HERE / f"random_w{wseed}_f{fseed}_{h}x{w}.npz",
            weight_seed=wseed, frame=frame, meta=meta.numpy(),
            upscale_tile0=whole.numpy(), upscale_tile32=tiled.numpy(),
        )



def bilinear(torch, F, folded_from_state):
    """The initial (head-zero) model equals 2x bilinear (tests/test_reference.py:56-61)."""
    state = random_folded_state(21)
    state["metadata_head.weight"][:] = 0
    state["metadata_head.bias"][:] = 0
    from aeisu_b200.synthetic import bilinear_base
    state["base_kernel"] = bilinear_base()
    src = torch.from_numpy(np.random.default_rng(22).random((1, 3, 12, 16), dtype=np.float32))
    with torch.inference_mode():
        out = folded_from_state(state)(src)
        bil = F.interpolate(src, scale_factor=2, mode="bilinear", align_corners=False)
    np.savez_compressed(HERE / "bilinear_identity.npz", source=src.numpy(), forward=out.numpy(),
                        bilinear=bil.numpy())



def trained(torch, ref, load_model, upscale, frame_chw):
    """Trained checkpoints (outputs only; the weights themselves are not stored)."""
    for ckpt, fseed, h, w, tile, deg in (("aeisu_area.pt", 200, 48, 64, 0, "area"),
                                          ("aeisu_area.pt", 0, 256, 256, 0, "area"),
                                          ("aeisu_bicubic.pt", 300, 150, 200, 64, "bicubic")):
        path = ref / "weights" / ckpt
        model = load_model(path, "cpu")
        frame = make_frame(fseed, h, w, deg)
        with torch.inference_mode():
            out = upscale(model, frame_chw(frame), tile)
        u8 = np.floor(out.permute(1, 2, 0).numpy() * 255 + 0.5).astype(np.uint8)
        extra = {}
        if h * w <= 64 * 64:
            extra["upscale_f32"] = out.numpy()
        else:
            cy, cx = h, w  # centre 128x128 HR window of the float output
            extra["window_f32"] = out[:, cy - 64:cy + 64, cx - 64:cx + 64].numpy()
            extra["window_origin"] = np.array([cy - 64, cx - 64])
        np.savez_compressed(
            HERE / f"{Path(ckpt).stem}_f{fseed}_{h}x{w}_t{tile}.npz",
            checkpoint=ckpt, checkpoint_sha256=sha256(path), frame=frame, tile=tile,
            degradation=deg, upscale_u8=u8, **extra)


def training(torch, load_model, upscale, frame_chw):
    """A train.py-style checkpoint (training coordinates not folded) through load_model, which
    folds it (aeisu/runtime.py:49-52).  The checkpoint is regenerated by the tests from the
    seeds with aeisu_b200.synthetic.seeded_training_state; the fixture keeps the reference's
    folded tensors and its upscale of one frame."""
    import tempfile
    from aeisu_b200.synthetic import seeded_training_state
    c = TRAINING
    state = seeded_training_state(random_folded_state(c["weight_seed"]), c["branch_seed"], c["branch_std"])
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(tmp) / "training.pt"
        torch.save({"model": {k: torch.from_numpy(v) for k, v in state.items()}, "basis_l1_scale": 0.5}, path)
        model = load_model(path, "cpu")
    folded = {k: v.numpy() for k, v in model.state_dict().items()}
    frame = make_frame(c["frame_seed"], c["h"], c["w"])
    with torch.inference_mode():
        out = upscale(model, frame_chw(frame), 0)
    np.savez_compressed(HERE / "training_checkpoint.npz", keys=np.array(list(state)),
                        folded_keys=np.array(list(folded)), **{f"folded.{k}": v for k, v in folded.items()},
                        frame=frame, upscale_f32=out.numpy(), **{k: np.array(v) for k, v in c.items()})


def tile256(torch, ref, load_model, upscale, frame_chw):
    """Config 4: the reference's tiled path (tile 256, 32-LR halos) on a 1920x1080 bicubic frame
    with aeisu_bicubic.pt.  The frame is regenerated by the tests from its seed (its SHA-256 is
    kept to confirm it); the float output is kept on the rows and columns around every tile seam
    (two on each side) and the uint8 output as per-row sums."""
    c = TILE256
    path = ref / "weights" / c["checkpoint"]
    model = load_model(path, "cpu")
    frame = make_frame(c["seed"], c["h"], c["w"], c["degradation"])
    with torch.inference_mode():
        out = upscale(model, frame_chw(frame), c["tile"]).numpy()
    rows, cols = seam_rows_cols(c["h"], c["w"], c["tile"])
    ridx = np.array([r + d for r in rows for d in (-2, -1, 0, 1)])
    cidx = np.array([x + d for x in cols for d in (-2, -1, 0, 1)])
    u8 = np.floor(out.transpose(1, 2, 0) * 255 + 0.5).astype(np.uint8)
    np.savez_compressed(
        HERE / "aeisu_bicubic_f400_1080x1920_t256.npz", checkpoint_sha256=sha256(path),
        frame_sha256=hashlib.sha256(frame.tobytes()).hexdigest(), seam_rows=np.array(rows),
        seam_cols=np.array(cols), row_index=ridx, col_index=cidx, rows_f32=out[:, ridx, :],
        cols_f32=out[:, :, cidx], u8_row_sums=u8.astype(np.int64).sum(axis=(1, 2)),
        **{k: np.array(v) for k, v in c.items()})


if __name__ == "__main__":
    main()

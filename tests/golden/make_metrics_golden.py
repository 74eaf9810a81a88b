"""Generate tests/golden/metrics_distortion.npz from the reference's own metric function.

Run where a checkout of the reference is available (its path via ``--reference``, or the
``AEISU_REFERENCE`` environment variable):

    python tests/golden/make_metrics_golden.py [--reference PATH]

It imports the reference's ``aeisu.metrics.distortion`` (aeisu/metrics.py:17-39) and records
y_mse, y_psnr and y_ssim for seeded synthetic image pairs: a target read as ``read_rgb`` gives
it (uint8 / 255) and a prediction that is the target plus noise, partly outside [0, 1] so that
the clamp matters, at several sizes and crops, including an exact match (PSNR = inf) and the
smallest size the crop allows.  The fixture is committed; tests never need the reference.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from aeisu_b200.synthetic import make_frame  # noqa: E402

# (seed, height, width, crop, noise)
CASES = (
    (500, 40, 52, 2, 0.02),
    (501, 15, 15, 2, 0.05),      # smallest frame crop 2 allows (11 + 2 * 2)
    (502, 33, 130, 0, 0.01),     # two window strips, no crop
    (503, 27, 31, 5, 0.10),
    (504, 24, 24, 2, 0.0),       # exact match: y_mse 0, y_psnr inf
    (505, 45, 100, 3, 0.03),
)


def pair(seed, h, w, noise):
    target = make_frame(seed, h, w).astype(np.float32).transpose(2, 0, 1) / np.float32(255)
    rng = np.random.default_rng(seed + 1)
    pred = target + rng.normal(0, noise, target.shape).astype(np.float32) if noise else target.copy()
    if noise:
        pred[:, :3, :3] += np.float32(0.5)   # some values above 1 (clamped by the metric)
        pred[:, -2:, -4:] -= np.float32(0.5)  # and below 0
    return np.ascontiguousarray(pred, np.float32), np.ascontiguousarray(target, np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AEISU_REFERENCE"),
                    help="checkout of the reference (default: $AEISU_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference checkout with --reference or AEISU_REFERENCE")
    sys.path.insert(0, args.reference)
    import torch
    from aeisu.metrics import distortion

    out = {}
    for i, (seed, h, w, crop, noise) in enumerate(CASES):
        p, t = pair(seed, h, w, noise)
        s = distortion(torch.from_numpy(p), torch.from_numpy(t), crop)
        out[f"pred{i}"] = p
        out[f"target{i}"] = t
        out[f"crop{i}"] = np.int64(crop)
        out[f"scores{i}"] = np.array([s["y_mse"], s["y_psnr"], s["y_ssim"]], np.float64)
    out["cases"] = np.int64(len(CASES))
    np.savez_compressed(HERE / "metrics_distortion.npz", **out)
    print(f"wrote {len(CASES)} cases to {HERE / 'metrics_distortion.npz'}")


if __name__ == "__main__":
    main()

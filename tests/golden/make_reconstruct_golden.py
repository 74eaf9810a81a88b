"""Generate the reconstruction forward/backward fixtures from the reference PyTorch code.

Run where a checkout of the reference is available (its path via ``--reference``, or the
``AEISU_REFERENCE`` environment variable):

    python tests/golden/make_reconstruct_golden.py [--reference PATH]

For each case it calls the reference's own ``aeisu.reconstruction.reconstruct`` (the function
train.py:99-103 differentiates) on seeded inputs with ``metadata``, ``base`` and ``basis``
requiring gradients, back-propagates a seeded upstream gradient, and records the output and the
three gradients (``None`` gradients are stored as empty arrays).  Metadata values are spread so
that every branch of the coefficient clamp (|v| <= 2, the soft ramp, the 2.5 ceiling) occurs.
The fixture is committed; tests never need the reference at run time.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# (name, batch, h, w, trim, gradient_stride, phase, seed)
CASES = (
    ("dense_t0", 1, 8, 12, 0, 1, 0, 11),
    ("ref_sampled", 1, 8, 12, 0, 4, 5, 12),      # the shape of tests/test_reference.py:79-99
    ("trim4_s2", 2, 16, 20, 4, 2, 3, 13),
    ("trim6_s3", 1, 18, 22, 6, 3, 7, 14),        # odd LR border (offset 3)
    ("trim32_s16", 1, 56, 48, 32, 16, 0, 15),    # the training recipe's trim and stride
    ("nograd_s0", 1, 10, 14, 0, 0, 0, 16),
    ("dense_24x34", 1, 24, 34, 0, 1, 0, 17),
    ("phase_wrap", 1, 20, 24, 4, 4, 37, 18),     # phase beyond stride**2 wraps
)


def inputs(b, h, w, seed):
    rng = np.random.default_rng(seed)
    src = rng.random((b, 3, h, w), dtype=np.float32)
    meta = (rng.standard_normal((b, 64, h // 2, w // 2)) * 1.5).astype(np.float32)
    pick = rng.random(meta.shape)
    meta[pick < 0.1] *= 6.0                      # soft ramp and ceiling
    meta[pick > 0.97] = np.float32(12.0) * np.sign(meta[pick > 0.97])   # the ceiling's bound
    base = (rng.standard_normal((25, 4)) * 0.05).astype(np.float32)
    basis = (rng.standard_normal((25, 16, 4)) * 0.05).astype(np.float32)
    return src, meta, base, basis


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AEISU_REFERENCE"),
                    help="checkout of the reference (default: $AEISU_REFERENCE)")
    ap.add_argument("--out", default=str(HERE / "reconstruct_grad.npz"))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference checkout with --reference or AEISU_REFERENCE")
    sys.path.insert(0, args.reference)
    import torch
    from aeisu.reconstruction import reconstruct

    torch.set_num_threads(4)
    record = {}
    for name, b, h, w, trim, stride, phase, seed in CASES:
        src, meta, base, basis = inputs(b, h, w, seed)
        off = trim // 2
        rng = np.random.default_rng(seed + 1000)
        grad = rng.standard_normal((b, 3, 2 * (h - 2 * off), 2 * (w - 2 * off))).astype(np.float32)
        tm, tb, tk = (torch.from_numpy(v.copy()).requires_grad_() for v in (meta, base, basis))
        out = reconstruct(torch.from_numpy(src), tm, tb, tk, trim=trim, gradient_stride=stride, phase=phase)
        out.backward(torch.from_numpy(grad))
        prefix = name + "/"
        record[prefix + "geom"] = np.array([b, h, w, trim, stride, phase], np.int64)
        for key, value in (("src", src), ("meta", meta), ("base", base), ("basis", basis), ("grad", grad)):
            record[prefix + key] = value
        record[prefix + "out"] = out.detach().numpy()
        for key, t in (("g_meta", tm), ("g_base", tb), ("g_basis", tk)):
            record[prefix + key] = t.grad.numpy() if t.grad is not None else np.zeros(0, np.float32)
    np.savez_compressed(args.out, **record)
    print(f"wrote {args.out}: {len(CASES)} cases")


if __name__ == "__main__":
    main()

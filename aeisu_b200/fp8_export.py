"""FP8 exporter: a SPYR8 v1 artifact (mixed FP8/FP16 route) from a folded FP32 checkpoint.

The reference ships the artifact format (optimized/native/src/neural/srcpyr/SrcPyrModel.cpp:
37-85 layout, 243-470 validation) and one exported file (adaptive_fp8.bin), not the tool that
made it; its supplement names the steps (paper/inverse_supersampling_supplement.tex:558-559):
per-output-channel E4M3 weight scales, activation scales calibrated on sample frames, and bias
correction of the FP8 layers.  This module restates them:

* weights: per output channel, scale = max|w| / 448 and E4M3 codes of w / scale (round to
  nearest even, as the reference artifact's codes are); FP16 copies for the FP16 layers;
* activation scales: the largest |x| of each quantised activation over the calibration frames,
  divided by 448, measured by the GPU's FP32 route (``aeisu_activation_stats``); optionally a
  coordinate search that tries smaller and larger scales one activation at a time and keeps
  the one with the best PSNR of the mixed route against FP32 on the same frames;
* bias correction (the FP8 layers compress, bottleneck 0-3, expand): ``bias_fp8 = bias +
  sum_k (w - dequant(w))[o, k] * mean(x_k)``, the expected output shift the weight rounding
  causes, from the calibration frames' input-channel means.

The tensor order, names and layouts are those of the reference artifact, so the result loads
with ``aeisu_open_spyr8`` (and the reference's own loader).

    python -m aeisu_b200.fp8_export CHECKPOINT.pt OUT.bin [--images A.png ...] [--synthetic N] [--search]
"""
from __future__ import annotations

import argparse
from pathlib import Path

import numpy as np

from . import spyr8
from .runtime import Model, _checkpoint_state

E4M3_MAX = 448.0
FP8_LAYERS = ("compress", "bottleneck0", "bottleneck1", "bottleneck2", "bottleneck3", "expand")
# offset of each FP8 layer's input channels in the means vector of aeisu_activation_stats
_MEAN_OFFSETS = {"compress": (0, 128), "bottleneck0": (128, 64), "bottleneck1": (192, 64),
                 "bottleneck2": (256, 64), "bottleneck3": (320, 64), "expand": (384, 64)}
_FOLDED_NAMES = {"project": "project_540", "compress": "compress_270", "expand": "expand_270",
                 "refine": "refine_540", "tail": "metadata_head"}


def load_folded_state(path):
    """(state dict of numpy arrays, basis_l1_scale) of a folded ``.pt`` checkpoint."""
    import torch  # checkpoint container only
    payload = torch.load(Path(path), map_location="cpu", weights_only=True)
    state = _checkpoint_state(payload)
    if any(".rep_low_u" in key for key in state):
        raise ValueError("training checkpoints must be folded first (export.py) before the FP8 export")
    scale = payload.get("basis_l1_scale", payload.get("config", {}).get("basis_l1_scale", 0.5)) \
        if isinstance(payload, dict) else 0.5
    return {k: (v.detach().cpu().numpy() if hasattr(v, "detach") else np.asarray(v)) for k, v in state.items()}, \
        float(scale)


def project_basis(raw, l1_scale=0.5):
    """reconstruction.py:8-12: centre each 25-tap vector of basis_raw [16,4,25], scale it to L1
    norm ``l1_scale`` (denominator clamped at 1e-6), permute to [25,16,4]."""
    raw = np.asarray(raw, np.float32)
    centred = raw - raw.mean(axis=-1, keepdims=True, dtype=np.float32)
    l1 = np.maximum(np.abs(centred).sum(axis=-1, keepdims=True, dtype=np.float32), np.float32(1e-6))
    return (centred * (np.float32(l1_scale) / l1)).transpose(2, 0, 1).astype(np.float32)


def layer_weights(state):
    """{SPYR8 layer name: (OIHW float32 weight, float32 bias)}; the grouped bottleneck layers
    hold cat(a_i, b_i) as the artifact stores them (SrcPyrModel.cpp:441-449)."""
    out = {}
    for name, key in _FOLDED_NAMES.items():
        out[name] = (np.asarray(state[f"{key}.weight"], np.float32), np.asarray(state[f"{key}.bias"], np.float32))
    for i in range(4):
        out[f"bottleneck{i}"] = (
            np.concatenate([state[f"bottleneck_270_a{i + 1}.weight"], state[f"bottleneck_270_b{i + 1}.weight"]]
                           ).astype(np.float32),
            np.concatenate([state[f"bottleneck_270_a{i + 1}.bias"], state[f"bottleneck_270_b{i + 1}.bias"]]
                           ).astype(np.float32))
    return out


def quantize_weight(w):
    """Per-output-channel E4M3: (codes, scales) with scale = max|w| / 448 (1e-12 floor)."""
    w = np.asarray(w, np.float32)
    scale = (np.maximum(np.abs(w).reshape(w.shape[0], -1).max(axis=1), 1e-12) / E4M3_MAX).astype(np.float32)
    codes = spyr8.e4m3_encode(w / scale.reshape(-1, *([1] * (w.ndim - 1))))
    return codes, scale


def bias_correction(w, codes, scale, means):
    """sum_k (w - dequant)[o, k] * mean_k per output channel o; k runs over the input channels
    of o's group (grouped layers: the weight holds CIN/groups inputs per output)."""
    err = (np.asarray(w, np.float64) - spyr8.e4m3_decode(codes).astype(np.float64)
           * scale.reshape(-1, 1, 1, 1)).sum(axis=(2, 3))   # [cout, cin_per_group]
    cout, cin = err.shape
    groups = len(means) // cin
    m = np.asarray(means, np.float64).reshape(groups, cin)
    return np.einsum("ok,ok->o", err, m[np.arange(cout) // (cout // groups)]).astype(np.float32)


def build_artifact(state, activation_scales, means=None, basis_l1_scale=0.5):
    """Serialise a SPYR8 v1 artifact from folded weights, activation scales (peak / 448) and,
    when given, the FP8 layers' input-channel means for bias correction."""
    scales = np.asarray(activation_scales, np.float32)
    if scales.shape != (10,) or not np.all(np.isfinite(scales)) or np.any(scales <= 0):
        raise ValueError("activation scales must be 10 positive finite values")
    lw = layer_weights(state)
    t = {"activation_scales": (scales, spyr8.VECTOR)}
    bias_fp8 = {}
    for name in spyr8.LAYER_NAMES:
        w, b = lw[name]
        codes, wscale = quantize_weight(w)
        t[f"{name}.weight_fp8"] = (codes, spyr8.OIHW)
        t[f"{name}.weight_fp16"] = (w.astype(np.float16), spyr8.OIHW)
        t[f"{name}.weight_scale"] = (wscale, spyr8.VECTOR)
        t[f"{name}.bias"] = (b, spyr8.VECTOR)
        t[f"{name}.prelu"] = (np.full(w.shape[0], 1.0 if name == "tail" else 0.1, np.float32), spyr8.VECTOR)
        corr = np.zeros_like(b)
        if means is not None and name in FP8_LAYERS:
            o, n = _MEAN_OFFSETS[name]
            corr = bias_correction(w, codes, wscale, np.asarray(means, np.float32)[o:o + n])
        bias_fp8[name] = (b + corr).astype(np.float32)
    for name in spyr8.LAYER_NAMES:
        t[f"{name}.bias_fp8"] = (bias_fp8[name], spyr8.VECTOR)
    t["adaptive_basis"] = (project_basis(state["basis_raw"], basis_l1_scale), spyr8.ADAPTIVE_BASIS)
    t["precision_guards"] = (np.zeros(2, np.float32), spyr8.VECTOR)
    t["adaptive_base"] = (np.asarray(state["base_kernel"], np.float32), spyr8.ADAPTIVE_BASIS)
    stencil = np.concatenate([np.asarray(state[k], np.float32).reshape(-1) for k in (
        "analysis_rgb_basis", "analysis_rgb_mix", "analysis_dx_rows", "analysis_dy_cols",
        "analysis_diag45", "analysis_diag135")])
    t["analysis_stencil"] = (stencil, spyr8.VECTOR)
    return spyr8.write_spyr8(t)


def calibrate(state, frames, device="cuda:0", basis_l1_scale=0.5):
    """(peaks[10], means[448]) of the FP32 route over uint8 frames [n,H,W,3] (or a list of
    frames of any sizes, measured one size at a time)."""
    model = Model.from_folded_state(state, device, "fp32", basis_l1_scale)
    try:
        if isinstance(frames, np.ndarray) and frames.ndim == 4:
            groups = [frames]
        else:
            groups = [np.asarray(f, np.uint8)[None] for f in frames]
        peaks = np.zeros(10, np.float32)
        sums = np.zeros(448, np.float64)
        weight = 0.0
        for g in groups:
            p, m = model.activation_stats(g)
            peaks = np.maximum(peaks, p)
            px = float(g.shape[0] * g.shape[1] * g.shape[2])
            sums += m.astype(np.float64) * px
            weight += px
        if not np.all(np.isfinite(peaks)):
            raise FloatingPointError("non-finite activation in the calibration frames")
        return peaks, (sums / weight).astype(np.float32)
    finally:
        model.close()


def _psnr(a, b):
    mse = float(np.mean((np.clip(a, 0, 1).astype(np.float64) - np.clip(b, 0, 1)) ** 2))
    return float("inf") if mse == 0 else 10 * np.log10(1.0 / mse)


def search_scales(state, scales, means, frames, device="cuda:0", basis_l1_scale=0.5,
                  factors=(0.5, 0.71, 1.41, 2.0), rounds=1):
    """Coordinate search over the ten activation scales: for each, try scale * f for f in
    `factors`, keep the best mean PSNR of the mixed route against the FP32 route on `frames`
    (uint8 [n,H,W,3]); `rounds` passes.  Returns (scales, PSNR before, PSNR after)."""
    frames = np.asarray(frames, np.uint8)
    src = frames.astype(np.float32).transpose(0, 3, 1, 2) / np.float32(255.0)
    fp32 = Model.from_folded_state(state, device, "fp32", basis_l1_scale)
    try:
        ref = fp32.upscale_f32(src, 0)
    finally:
        fp32.close()

    def score(s):
        m = Model.from_spyr8_bytes(build_artifact(state, s, means, basis_l1_scale), device, "mixed")
        try:
            return _psnr(m.upscale_f32(src, 0), ref)
        finally:
            m.close()

    best = np.asarray(scales, np.float32).copy()
    best_score = first = score(best)
    for _ in range(rounds):
        for k in range(10):
            for f in factors:
                trial = best.copy()
                trial[k] = np.float32(best[k] * f)
                s = score(trial)
                if s > best_score:
                    best, best_score = trial, s
    return best, first, best_score


def export_spyr8(checkpoint, frames, device="cuda:0", search=False, out=None):
    """Calibrate the folded checkpoint on uint8 frames and return (and optionally write to
    `out`) the SPYR8 artifact bytes."""
    state, l1 = load_folded_state(checkpoint)
    peaks, means = calibrate(state, frames, device, l1)
    scales = np.maximum(peaks, 1e-6) / np.float32(E4M3_MAX)
    if search:
        scales, _, _ = search_scales(state, scales, means, frames, device, l1)
    data = build_artifact(state, scales, means, l1)
    if out is not None:
        Path(out).write_bytes(data)
    return data


def _read_u8(path):
    from PIL import Image
    with Image.open(path) as image:
        return np.array(image.convert("RGB"), dtype=np.uint8, copy=True)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("checkpoint")
    ap.add_argument("out")
    ap.add_argument("--images", nargs="*", default=[], help="calibration images (PNG/JPEG)")
    ap.add_argument("--synthetic", type=int, default=0, help="add N seeded procedural 256x256 scenes")
    ap.add_argument("--search", action="store_true", help="coordinate search of the activation scales")
    ap.add_argument("--device", default="cuda:0")
    args = ap.parse_args(argv)
    frames = [_read_u8(p) for p in args.images]
    if args.synthetic:
        from .synthetic import make_frames
        frames += list(make_frames(9000, args.synthetic, 256, 256))
    if not frames:
        ap.error("give calibration frames (--images and/or --synthetic)")
    same = len({f.shape for f in frames}) == 1
    batch = np.stack(frames) if same else frames
    if args.search and not same:
        ap.error("--search needs frames of one size")
    data = export_spyr8(args.checkpoint, batch, args.device, args.search, args.out)
    print(f"{args.out}: {len(data)} bytes, sha256 {spyr8.checksum(data)}")


if __name__ == "__main__":
    main()

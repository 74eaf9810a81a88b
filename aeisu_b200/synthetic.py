"""Seeded synthetic workloads: procedural test frames and random-init folded weights.

The reference benchmarks on private or external image sets; these seeded scenes
stand in for them with the shapes, value range and degradations the workload
definitions name: a 2x-resolution procedural scene in [0,1] sRGB (40 polygons with
flat or linear-gradient fills, 10 sinusoidal texture patches with 2-32 px periods,
20 anti-aliased 1-2 px lines), rounded to uint8, then degraded to the input
resolution by either the 2x2 integer area average ``(sum+2)//4`` (the convention of
research/archival_sources/paper_bench/common.py:40-48) or a 2x bicubic (a=-0.5)
downsample.

``random_folded_state`` builds random weights with the folded AEISU layout
(aeisu/model.py:554-583) for parity tests and for runs without a trained checkpoint.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def _fill_polygon(canvas, verts, color_fn):
    """Even-odd scanline fill of one polygon; ``color_fn(ys, xs)`` gives [n,3] colours."""
    h, w, _ = canvas.shape
    y0 = max(int(np.floor(verts[:, 1].min())), 0)
    y1 = min(int(np.ceil(verts[:, 1].max())) + 1, h)
    x0 = max(int(np.floor(verts[:, 0].min())), 0)
    x1 = min(int(np.ceil(verts[:, 0].max())) + 1, w)
    if y1 <= y0 or x1 <= x0:
        return
    ys = np.arange(y0, y1, dtype=np.float64) + 0.5
    a = verts
    b = np.roll(verts, -1, axis=0)
    ay, by = a[:, 1][None, :], b[:, 1][None, :]
    yy = ys[:, None]
    crosses = ((ay <= yy) & (by > yy)) | ((by <= yy) & (ay > yy))
    with np.errstate(divide="ignore", invalid="ignore"):
        t = (yy - ay) / (by - ay)
    xc = a[:, 0][None, :] + t * (b[:, 0] - a[:, 0])[None, :]
    # a pixel (centre x+0.5) is inside when an odd number of crossings lie left of it
    col = np.clip(np.ceil(xc - 0.5).astype(np.int64) - x0, 0, x1 - x0)
    toggles = np.zeros((y1 - y0, x1 - x0 + 1), np.int32)
    rows = np.broadcast_to(np.arange(y1 - y0)[:, None], col.shape)
    np.add.at(toggles, (rows[crosses], col[crosses]), 1)
    inside = (np.cumsum(toggles[:, :-1], axis=1) & 1).astype(bool)
    iy, ix = np.nonzero(inside)
    if iy.size:
        canvas[iy + y0, ix + x0] = color_fn(iy + y0 + 0.5, ix + x0 + 0.5)


def procedural_scene(h, w, rng):
    """Render one [h, w, 3] float32 scene in [0, 1]."""
    canvas = np.empty((h, w, 3), F32)
    c0, c1 = rng.random(3), rng.random(3)
    gy = np.linspace(0, 1, h, dtype=F32)[:, None, None]
    canvas[:] = (c0 * (1 - gy) + c1 * gy).astype(F32)
    scale = min(h, w)
    for _ in range(40):
        n = int(rng.integers(3, 8))
        cx, cy = rng.random() * w, rng.random() * h
        radius = scale * (0.04 + 0.22 * rng.random())
        ang = np.sort(rng.random(n)) * 2 * np.pi
        rad = radius * (0.5 + 0.5 * rng.random(n))
        verts = np.stack([cx + rad * np.cos(ang), cy + rad * np.sin(ang)], axis=1)
        col_a = rng.random(3)
        if rng.random() < 0.5:
            def color_fn(ys, xs, col_a=col_a):
                return np.broadcast_to(col_a.astype(F32), (ys.size, 3))
        else:
            col_b = rng.random(3)
            theta = rng.random() * 2 * np.pi
            d = np.array([np.cos(theta), np.sin(theta)])

            def color_fn(ys, xs, col_a=col_a, col_b=col_b, d=d, cx=cx, cy=cy, radius=radius):
                t = ((xs - cx) * d[0] + (ys - cy) * d[1]) / (2 * radius) + 0.5
                t = np.clip(t, 0, 1)[:, None]
                return (col_a * (1 - t) + col_b * t).astype(F32)
        _fill_polygon(canvas, verts, color_fn)
    for _ in range(10):
        ph, pw = int(scale * (0.05 + 0.2 * rng.random())) + 2, int(scale * (0.05 + 0.2 * rng.random())) + 2
        y0, x0 = int(rng.integers(0, max(h - ph, 1))), int(rng.integers(0, max(w - pw, 1)))
        ph, pw = min(ph, h - y0), min(pw, w - x0)
        period = 2.0 + 30.0 * rng.random()
        theta = rng.random() * np.pi
        phase = rng.random() * 2 * np.pi
        yy, xx = np.mgrid[0:ph, 0:pw].astype(F32)
        wave = np.sin(2 * np.pi * (xx * np.cos(theta) + yy * np.sin(theta)) / period + phase)
        base, amp = rng.random(3), 0.5 * rng.random(3)
        canvas[y0:y0 + ph, x0:x0 + pw] = np.clip(base + amp * wave[..., None], 0, 1).astype(F32)
    for _ in range(20):
        p0 = np.array([rng.random() * w, rng.random() * h])
        length = scale * (0.1 + 0.5 * rng.random())
        theta = rng.random() * 2 * np.pi
        p1 = p0 + length * np.array([np.cos(theta), np.sin(theta)])
        width = 1.0 + rng.random()
        color = rng.random(3).astype(F32)
        lx0 = max(int(min(p0[0], p1[0]) - 2), 0)
        lx1 = min(int(max(p0[0], p1[0]) + 3), w)
        ly0 = max(int(min(p0[1], p1[1]) - 2), 0)
        ly1 = min(int(max(p0[1], p1[1]) + 3), h)
        if lx1 <= lx0 or ly1 <= ly0:
            continue
        yy, xx = np.mgrid[ly0:ly1, lx0:lx1].astype(np.float64) + 0.5
        d = p1 - p0
        t = np.clip(((xx - p0[0]) * d[0] + (yy - p0[1]) * d[1]) / max(d @ d, 1e-9), 0, 1)
        dist = np.hypot(xx - (p0[0] + t * d[0]), yy - (p0[1] + t * d[1]))
        cover = np.clip(width / 2 + 0.5 - dist, 0, 1).astype(F32)[..., None]
        region = canvas[ly0:ly1, lx0:lx1]
        canvas[ly0:ly1, lx0:lx1] = region * (1 - cover) + color * cover
    return canvas


def to_u8(image):
    return np.floor(np.clip(image, 0, 1) * 255 + 0.5).astype(np.uint8)


def area_downsample(hr_u8):
    """2x2 integer box average with round-half-up: (sum + 2) // 4."""
    h, w, c = hr_u8.shape
    s = hr_u8[:h - h % 2, :w - w % 2].astype(np.uint16).reshape(h // 2, 2, w // 2, 2, c).sum((1, 3))
    return ((s + 2) // 4).astype(np.uint8)


def _cubic(x, a=-0.5):
    x = np.abs(x)
    return np.where(x <= 1, ((a + 2) * x - (a + 3)) * x * x + 1,
                    np.where(x < 2, ((a * x - 5 * a) * x + 8 * a) * x - 4 * a, 0.0))


def bicubic_downsample(hr_u8):
    """Antialiased 2x bicubic (a=-0.5) downsample with edge clamping, rounded to uint8."""
    hr = hr_u8.astype(np.float64)
    taps = np.arange(-3, 5)                               # HR offsets around 2j
    wts = _cubic((taps + 0.5 - 1.0) / 2.0)
    wts = wts / wts.sum()

    def along(a, axis):
        n = a.shape[axis] // 2
        idx = np.clip(2 * np.arange(n)[:, None] + taps[None, :], 0, a.shape[axis] - 1)
        g = np.take(a, idx, axis=axis)                   # inserts [n, 8] at axis
        return np.tensordot(g, wts, axes=([axis + 1], [0]))

    out = along(along(hr, 0), 1)
    return np.clip(np.floor(out + 0.5), 0, 255).astype(np.uint8)


def make_frame(seed, height, width, degradation="area"):
    """One seeded uint8 [height, width, 3] input frame."""
    rng = np.random.default_rng(seed)
    hr = to_u8(procedural_scene(2 * height, 2 * width, rng))
    if degradation == "area":
        return area_downsample(hr)
    if degradation == "bicubic":
        return bicubic_downsample(hr)
    raise ValueError(f"unknown degradation {degradation!r}")


def make_frames(seed, count, height, width, degradation="area"):
    out = np.empty((count, height, width, 3), np.uint8)
    for i in range(count):
        out[i] = make_frame(seed + i, height, width, degradation)
    return out


# ---- random-init weights with the folded checkpoint layout ----------------------

_CONVS = (
    ("project_540", 32, 32, 1),
    ("compress_270", 128, 64, 1),
    *((f"bottleneck_270_{b}{i}", 32, 32, 3) for b in ("a", "b") for i in range(1, 5)),
    ("expand_270", 64, 128, 1),
    ("refine_540", 32, 64, 3),
    ("metadata_head", 64, 64, 1),
)


def bilinear_base():
    """The exact 2x bilinear filter as [25 taps, 4 phases] (phase order TL, TR, BL, BR)."""
    base = np.zeros((25, 4), F32)
    q1, q3, q9 = 1 / 16, 3 / 16, 9 / 16
    for phase in range(4):
        oy, ox = phase >> 1, phase & 1
        for dy, wy in ((0, 0.25 if oy == 0 else 0.75), (1, 0.75 if oy == 0 else 0.25)):
            for dx, wx in ((0, 0.25 if ox == 0 else 0.75), (1, 0.75 if ox == 0 else 0.25)):
                ty, tx = 1 + oy + dy, 1 + ox + dx
                base[ty * 5 + tx, phase] = wy * wx
    assert sorted(set(np.round(base[base > 0] * 16).astype(int).tolist())) == [1, 3, 9]
    del q1, q3, q9
    return base


def random_folded_state(seed, coeff_gain=1.0):
    """Random folded weights (34 tensors, 115,996 values) for seeded parity tests."""
    rng = np.random.default_rng(seed)
    st = {}
    st["analysis_rgb_basis"] = (np.eye(3) + rng.normal(0, 0.1, (3, 3))).astype(F32)
    st["analysis_rgb_mix"] = (np.array([0.2126, 0.7152, 0.0722]) + rng.normal(0, 0.05, 3)).astype(F32)
    st["analysis_dx_rows"] = (np.array([0.125, 0.25, 0.125]) * 4 + rng.normal(0, 0.2, 3)).astype(F32)
    st["analysis_dy_cols"] = (np.array([0.125, 0.25, 0.125]) * 4 + rng.normal(0, 0.2, 3)).astype(F32)
    st["analysis_diag45"] = (np.array([0.25, 0.125, 0.125]) * 4 + rng.normal(0, 0.2, 3)).astype(F32)
    st["analysis_diag135"] = (np.array([0.25, 0.125, 0.125]) * 4 + rng.normal(0, 0.2, 3)).astype(F32)
    st["base_kernel"] = (bilinear_base() + rng.normal(0, 0.01, (25, 4))).astype(F32)
    st["basis_raw"] = rng.normal(0, 0.05, (16, 4, 25)).astype(F32)
    gain = np.sqrt(2.0 / (1 + 0.01))
    for name, cin, cout, k in _CONVS:
        fan_in = cin * k * k
        std = gain / np.sqrt(fan_in)
        if name == "metadata_head":
            std = coeff_gain * 2.0 / np.sqrt(fan_in)
        st[f"{name}.weight"] = rng.normal(0, std, (cout, cin, k, k)).astype(F32)
        st[f"{name}.bias"] = rng.normal(0, 0.05, cout).astype(F32)
    return st


def seeded_training_state(folded, seed, std=0.01):
    """A training checkpoint state (the AEISU layout, aeisu/model.py:37-168) whose main tensors
    are the given folded ones and whose training-only coordinates (low-rank, structural,
    template and mixed-bank branches, analysis gains) are N(0, std) draws from a seeded
    generator, in state_dict order; folding it changes every deployed tensor."""
    from .fold import training_shapes
    rng = np.random.default_rng(seed)
    out = {}
    for key, shape in training_shapes().items():
        out[key] = (np.array(folded[key], F32) if key in folded
                    else rng.normal(0, std, shape).astype(F32))
    return out


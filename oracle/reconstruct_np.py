"""FP32 numpy restatement of the reference's training-time reconstruction (TEST ORACLE ONLY).

Only tests may import this module.  It restates ``reconstruct`` of aeisu/reconstruction.py:29-83
with its ``trim``, ``gradient_stride`` and ``phase`` options, and the gradients autograd takes
through it (the reference has no hand-written backward: train.py:99-103 calls ``loss.backward()``
on this graph).  Paths are relative to the AELabs42/AEISU checkout.

Gradient semantics (reconstruction.py:56-78):

* coefficient gradients are always dense: ``weights = base + einsum(coeff, basis)`` routes every
  pixel's filter gradient into its 16 coefficients through the clamp of reconstruction.py:15-17;
* ``gradient_stride == 1``: base and basis gradients sum over every core pixel;
* ``gradient_stride > 1``: they sum only over the pixels with ``y % s == phase // s`` and
  ``x % s == phase % s`` (core coordinates, ``phase`` taken mod ``s**2``), each scaled by ``s**2``;
* ``gradient_stride == 0``: base and basis receive no gradient (``None``).
"""
from __future__ import annotations

import numpy as np

from .aeisu_np import F32, coefficient_clamp, unpack_coefficients


def check_geometry(src_shape, meta_shape, trim, gradient_stride=1, phase=0):
    """reconstruction.py:37-52: the argument checks, in the reference's order and words."""
    if len(src_shape) != 4 or src_shape[1] != 3:
        raise ValueError("Expected NCHW RGB source")
    if trim < 0 or trim % 2 or (trim and trim < 4):
        raise ValueError("trim must be zero or an even HR border of at least 4 pixels")
    if gradient_stride < 0 or phase < 0:
        raise ValueError("gradient_stride and phase must be nonnegative")
    b, _, h, w = src_shape
    off = trim // 2
    ch, cw = h - 2 * off, w - 2 * off
    # odd h or w make the reference's reshape of the unpacked coefficients fail as well
    if ch <= 0 or cw <= 0 or tuple(meta_shape) != (b, 64, h // 2, w // 2) or h % 2 or w % 2:
        raise ValueError("Source, metadata or trim geometry is invalid")
    return off, ch, cw


def _local(src, off, ch, cw):
    """reconstruction.py:53-57: the 5x5 neighbourhood source of the core (replicate pad at trim 0)."""
    if off:
        return src[:, :, off - 2:off + ch + 2, off - 2:off + cw + 2]
    return np.pad(src, ((0, 0), (0, 0), (2, 2), (2, 2)), mode="edge")


def _core_coefficients(meta, off, ch, cw):
    """Raw (unclamped) and clamped coefficients of the core pixels, [B, ch*cw, 16]."""
    b, _, hh, ww = meta.shape
    raw = meta.reshape(b, 4, 16, hh, ww).transpose(0, 2, 1, 3, 4).reshape(b, 16, 2, 2, hh, ww)
    raw = raw.transpose(0, 1, 4, 2, 5, 3).reshape(b, 16, 2 * hh, 2 * ww)     # pixel_shuffle
    raw = raw[:, :, off:off + ch, off:off + cw]
    raw = np.ascontiguousarray(raw.transpose(0, 2, 3, 1)).reshape(b, ch * cw, 16).astype(F32)
    return raw, coefficient_clamp(raw)


def reconstruct(src, meta, base, basis, trim=0):
    """reconstruction.py:29-83 forward: unclipped 2x RGB of the core, [B, 3, 2ch, 2cw]."""
    src = np.asarray(src, F32)
    off, ch, cw = check_geometry(src.shape, meta.shape, trim)
    b = src.shape[0]
    _, cf = _core_coefficients(np.asarray(meta, F32), off, ch, cw)
    local = _local(src, off, ch, cw)
    rgb = np.zeros((b, 3, ch, cw, 4), F32)
    for ky in range(5):
        for kx in range(5):
            t = ky * 5 + kx
            wt = (cf @ basis[t] + base[t]).reshape(b, ch, cw, 4)
            for c in range(3):
                rgb[:, c] += local[:, c, ky:ky + ch, kx:kx + cw, None] * wt
    out = rgb.reshape(b, 3, ch, cw, 2, 2).transpose(0, 1, 2, 4, 3, 5).reshape(b, 3, 2 * ch, 2 * cw)
    return np.ascontiguousarray(out, F32)


def sample_mask(ch, cw, gradient_stride, phase):
    """reconstruction.py:60-66: per-pixel weight of the base/basis gradient, [ch*cw]."""
    s = gradient_stride
    if s <= 1:
        return np.ones(ch * cw, F32)
    ph = phase % (s * s)
    yy = np.arange(ch)[:, None]
    xx = np.arange(cw)[None, :]
    m = (yy % s == ph // s) & (xx % s == ph % s)
    return (m.astype(F32) * F32(s * s)).reshape(-1)


def clamp_grad(raw, g):
    """Gradient of coefficient_clamp (reconstruction.py:15-17) as autograd forms it: 1 where
    |v| <= 2; else 0.05 while 2 + 0.05 (|v| - 2) <= 2.5 (clamp(max=) passes its bound); else 0."""
    mag = np.abs(raw)
    soft = F32(2) + F32(0.05) * (mag - F32(2))
    return np.where(mag <= 2, g, np.where(soft <= F32(2.5), F32(0.05) * g, F32(0))).astype(F32)


def reconstruct_backward(src, meta, base, basis, grad, trim=0, gradient_stride=1, phase=0):
    """Gradients of ``(reconstruct(...) * grad).sum()`` with respect to metadata, base and basis.

    Returns (grad_meta [B,64,h/2,w/2], grad_base [25,4] or None, grad_basis [25,16,4] or None).
    """
    src = np.asarray(src, F32)
    meta = np.asarray(meta, F32)
    off, ch, cw = check_geometry(src.shape, meta.shape, trim, gradient_stride, phase)
    b, _, h, w = src.shape
    n = ch * cw
    raw, cf = _core_coefficients(meta, off, ch, cw)
    local = _local(src, off, ch, cw)
    # g[b, c, y, x, phase], phase = 2i + j of HR pixel (2y + i, 2x + j)
    g = np.asarray(grad, F32).reshape(b, 3, ch, 2, cw, 2).transpose(0, 1, 2, 4, 3, 5).reshape(b, 3, n, 4)
    mask = sample_mask(ch, cw, gradient_stride, phase)
    gcoef = np.zeros((b, n, 16), F32)
    gbase = np.zeros((25, 4), F32)
    gbasis = np.zeros((25, 16, 4), F32)
    mc = cf * mask[None, :, None]
    for ky in range(5):
        for kx in range(5):
            t = ky * 5 + kx
            patch = local[:, :, ky:ky + ch, kx:kx + cw].reshape(b, 3, n)
            gw = (patch[..., None] * g).sum(axis=1, dtype=F32)          # [b, n, 4] filter gradient
            gcoef += gw @ basis[t].T                                     # [b, n, 16]
            if gradient_stride:
                gbase[t] = (gw * mask[None, :, None]).sum(axis=(0, 1), dtype=F32)
                gbasis[t] = np.einsum("bnk,bnp->kp", mc, gw).astype(F32)
    gv = clamp_grad(raw, gcoef)                                           # [b, n, 16]
    full = np.zeros((b, 16, h, w), F32)
    full[:, :, off:off + ch, off:off + cw] = gv.reshape(b, ch, cw, 16).transpose(0, 3, 1, 2)
    # inverse of unpack_coefficients: meta channel parity*16 + k at (Y/2, X/2)
    gm = full.reshape(b, 16, h // 2, 2, w // 2, 2).transpose(0, 3, 5, 1, 2, 4).reshape(b, 64, h // 2, w // 2)
    if not gradient_stride:
        return np.ascontiguousarray(gm), None, None
    return np.ascontiguousarray(gm), gbase, gbasis


__all__ = ["check_geometry", "reconstruct", "reconstruct_backward", "sample_mask", "clamp_grad",
           "unpack_coefficients"]

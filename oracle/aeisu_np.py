"""FP32 numpy restatement of the reference AEISU inference path (TEST ORACLE ONLY).

Only tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
may import this module.  Each function cites the reference file:line it restates
(paths relative to the AELabs42/AEISU checkout).

Layouts follow the reference: activations are NCHW float32, convolution weights
OIHW, ``basis`` is the projected [25 taps, 16 components, 4 phases] bank.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
SLOPE = F32(0.1)  # aeisu/reparameterization.py:8 LEAKY_RELU_SLOPE

# aeisu/model.py:20-27 CONVOLUTIONS (name, in, out, kernel)
CONVOLUTIONS = (
    ("project_540", 32, 32, 1),
    ("compress_270", 128, 64, 1),
    *((f"bottleneck_270_{b}{i}", 32, 32, 3) for b in ("a", "b") for i in range(1, 5)),
    ("expand_270", 64, 128, 1),
    ("refine_540", 32, 64, 3),
    ("metadata_head", 64, 64, 1),
)

# FoldedAEISU.state_dict() order (aeisu/model.py:554-583); 34 tensors, 115,996 values.
STATE_SHAPES = (
    ("analysis_rgb_basis", (3, 3)),
    ("analysis_rgb_mix", (3,)),
    ("analysis_dx_rows", (3,)),
    ("analysis_dy_cols", (3,)),
    ("analysis_diag45", (3,)),
    ("analysis_diag135", (3,)),
    ("base_kernel", (25, 4)),
    ("basis_raw", (16, 4, 25)),
    *(item for name, cin, cout, k in CONVOLUTIONS
      for item in ((f"{name}.weight", (cout, cin, k, k)), (f"{name}.bias", (cout,)))),
)


def leaky(x):
    """F.leaky_relu(x, 0.1) (aeisu/model.py:202-203); max(x, 0.1x) is the same map for slope < 1."""
    t = np.multiply(x, SLOPE, dtype=F32)
    return np.maximum(x, t, out=t)


def pixel_unshuffle(x, r=2):
    """F.pixel_unshuffle: out[c*r*r + i*r + j, y, x] = in[c, r*y+i, r*x+j]."""
    b, c, h, w = x.shape
    return (x.reshape(b, c, h // r, r, w // r, r).transpose(0, 1, 3, 5, 2, 4)
            .reshape(b, c * r * r, h // r, w // r))


def pixel_shuffle(x, r=2):
    """F.pixel_shuffle: out[c, r*y+i, r*x+j] = in[c*r*r + i*r + j, y, x]."""
    b, c, h, w = x.shape
    co = c // (r * r)
    return (x.reshape(b, co, r, r, h, w).transpose(0, 1, 4, 2, 5, 3)
            .reshape(b, co, h * r, w * r))


def conv2d_nhwc(x, weight, bias, groups=1):
    """nn.Conv2d(padding=k//2, zero padding) on NHWC float32 data as float32 GEMMs.

    3x3: the zero-padded input is flattened row-major with row pitch W+2, so tap (ky, kx)
    of every output pixel is the contiguous slice shifted by ky*(W+2)+kx; each tap is one
    GEMM, accumulated, and the two pitch-padding columns are dropped at the end."""
    b, h, w, c = x.shape
    cout, cin_g, k, _ = weight.shape
    cout_g = cout // groups
    if k == 1:
        out = np.empty((b, h * w, cout), F32)
        xf = x.reshape(b, h * w, c)
        for g in range(groups):
            wg = weight[g * cout_g:(g + 1) * cout_g, :, 0, 0]
            out[:, :, g * cout_g:(g + 1) * cout_g] = xf[:, :, g * cin_g:(g + 1) * cin_g] @ wg.T
        out += bias
        return out.reshape(b, h, w, cout)
    pitch = w + 2
    flat = np.pad(x, ((0, 0), (1, 1), (1, 1), (0, 0))).reshape(b, (h + 2) * pitch, c)
    n = (h - 1) * pitch + w
    out = np.zeros((b, h * pitch, cout), F32)
    for g in range(groups):
        cs = slice(g * cin_g, (g + 1) * cin_g)
        os_ = slice(g * cout_g, (g + 1) * cout_g)
        for ky in range(3):
            for kx in range(3):
                off = ky * pitch + kx
                out[:, :n, os_] += flat[:, off:off + n, cs] @ weight[os_, :, ky, kx].T
    out = out.reshape(b, h, pitch, cout)[:, :, :w]
    return out + bias


def conv2d(x, weight, bias, groups=1):
    """NCHW wrapper of conv2d_nhwc."""
    return np.ascontiguousarray(
        conv2d_nhwc(np.ascontiguousarray(x.transpose(0, 2, 3, 1)), weight, bias, groups).transpose(0, 3, 1, 2))


def feature8(src, st):
    """_rgb_to_feature8 (aeisu/model.py:273-341): learned RGB, luma, 4 directional maps.

    Evaluated as separate float32 multiplies and adds in the reference's order
    (no fused multiply-add), as the PyTorch elementwise ops are.
    """
    r, g, b = src[:, 0:1], src[:, 1:2], src[:, 2:3]
    m = st["analysis_rgb_basis"]
    lr = [(r * m[i, 0] + g * m[i, 1]) + b * m[i, 2] for i in range(3)]
    mix = st["analysis_rgb_mix"]
    y = (r * mix[0] + g * mix[1]) + b * mix[2]
    yp = np.pad(y, ((0, 0), (0, 0), (1, 1), (1, 1)), mode="edge")
    ul, uc, ur = yp[:, :, :-2, :-2], yp[:, :, :-2, 1:-1], yp[:, :, :-2, 2:]
    cl, cr = yp[:, :, 1:-1, :-2], yp[:, :, 1:-1, 2:]
    dl, dc, dr = yp[:, :, 2:, :-2], yp[:, :, 2:, 1:-1], yp[:, :, 2:, 2:]
    hmid = cr - cl
    vmid = dc - uc
    a = st["analysis_dx_rows"]
    dx = ((ur - ul) * a[0] + hmid * a[1]) + (dr - dl) * a[2]
    a = st["analysis_dy_cols"]
    dy = ((dl - ul) * a[0] + vmid * a[1]) + (dr - ur) * a[2]
    a = st["analysis_diag45"]
    d45 = ((dr - ul) * a[0] + vmid * a[1]) + hmid * a[2]
    a = st["analysis_diag135"]
    d135 = ((ur - dl) * a[0] - vmid * a[1]) + hmid * a[2]
    return np.concatenate(lr + [y, dx, dy, d45, d135], axis=1).astype(F32)


def controller(src, st):
    """AEISU._controller (aeisu/model.py:473-492) -> metadata [B,64,H/2,W/2]."""
    if src.ndim != 4 or src.shape[1] != 3:
        raise ValueError("Expected source RGB [B,3,H,W]")
    if src.shape[2] % 4 or src.shape[3] % 4:
        raise ValueError("Source H/W must be divisible by 4")

    # Same graph, computed channels-last; the unshuffle/shuffle index maps are those of
    # F.pixel_unshuffle / F.pixel_shuffle (channel c*4 + i*2 + j <-> pixel offset (i, j)).
    def conv(name, x, groups=1):
        return conv2d_nhwc(x, st[f"{name}.weight"], st[f"{name}.bias"], groups)

    def unshuffle(x):
        b, h, w, c = x.shape
        return (x.reshape(b, h // 2, 2, w // 2, 2, c).transpose(0, 1, 3, 5, 2, 4)
                .reshape(b, h // 2, w // 2, c * 4))

    def shuffle(x):
        b, h, w, c4 = x.shape
        c = c4 // 4
        return (x.reshape(b, h, w, c, 2, 2).transpose(0, 1, 4, 2, 5, 3).reshape(b, h * 2, w * 2, c))

    feat = np.ascontiguousarray(feature8(src, st).transpose(0, 2, 3, 1))
    enc540 = leaky(conv("project_540", unshuffle(feat)))
    enc270 = leaky(conv("compress_270", unshuffle(enc540)))
    a, b = np.ascontiguousarray(enc270[..., :32]), np.ascontiguousarray(enc270[..., 32:])
    for i in range(1, 5):
        a = leaky(conv(f"bottleneck_270_a{i}", a))
        b = leaky(conv(f"bottleneck_270_b{i}", b))
    up540 = shuffle(leaky(conv("expand_270", np.concatenate((a, b), axis=-1))))
    dec540 = leaky(conv("refine_540", enc540 + up540))
    return np.ascontiguousarray(conv("metadata_head", dec540).transpose(0, 3, 1, 2))


def project_basis(raw, scale=0.5):
    """reconstruction.py:8-12: zero-DC, L1=scale, permuted to [tap, component, phase]."""
    raw = raw.astype(F32)
    centered = raw - raw.mean(axis=-1, keepdims=True, dtype=F32)
    den = np.maximum(np.abs(centered).sum(axis=-1, keepdims=True, dtype=F32), F32(1e-6))
    normalized = centered * (F32(scale) / den)
    return np.ascontiguousarray(normalized.transpose(2, 0, 1)).astype(F32)


def coefficient_clamp(v):
    """reconstruction.py:15-17: |v|<=2 passes, else sign*min(2.5, 2+0.05(|v|-2))."""
    v = np.asarray(v, F32)
    mag = np.abs(v)
    soft = np.minimum(F32(2) + F32(0.05) * (mag - F32(2)), F32(2.5))
    return np.where(mag <= 2, v, np.sign(v) * soft).astype(F32)


def unpack_coefficients(meta):
    """reconstruction.py:20-26: LR-parity-major channels -> [B,16,2h,2w] clamped."""
    b, c, h, w = meta.shape
    if c != 64:
        raise ValueError("Expected 64 packed coefficient channels")
    packed = meta.reshape(b, 4, 16, h, w).transpose(0, 2, 1, 3, 4).reshape(b, 64, h, w)
    # the clamp is elementwise, so it is applied before the (copying) shuffle
    return pixel_shuffle(coefficient_clamp(packed))


def reconstruct(src, meta, base, basis):
    """reconstruction.py:29-83 with trim=0, gradient_stride=1: unclipped 2x RGB."""
    b, _, h, w = src.shape
    if meta.shape != (b, 64, h // 2, w // 2):
        raise ValueError("Source, metadata or trim geometry is invalid")
    coeff = unpack_coefficients(meta)                        # [B,16,h,w]
    cf = np.ascontiguousarray(coeff.transpose(0, 2, 3, 1)).reshape(b, h * w, 16)
    local = np.pad(src, ((0, 0), (0, 0), (2, 2), (2, 2)), mode="edge")
    # rgb[b, c, y, x, phase] = sum_t patch_t[c] * (base[t, phase] + sum_k coeff_k * basis[t, k, phase]),
    # taps t = 5*ky + kx of the replicate-padded 5x5 neighbourhood (unfold order)
    rgb = np.zeros((b, 3, h, w, 4), F32)
    for ky in range(5):
        for kx in range(5):
            t = ky * 5 + kx
            wt = (cf @ basis[t] + base[t]).reshape(b, h, w, 4)
            for c in range(3):
                rgb[:, c] += local[:, c, ky:ky + h, kx:kx + w, None] * wt
    out = rgb.reshape(b, 3, h, w, 2, 2).transpose(0, 1, 2, 4, 3, 5).reshape(b, 3, 2 * h, 2 * w)
    return np.ascontiguousarray(out, F32)


class FoldedModel:
    """Deployed parameters of FoldedAEISU (aeisu/model.py:554-596) as numpy arrays."""

    def __init__(self, state, basis_l1_scale=0.5, basis=None):
        """``basis``: an already projected [25,16,4] bank (SPYR8 artifacts store it so);
        then ``basis_raw`` may be absent from ``state``."""
        keys = [(k, s) for k, s in STATE_SHAPES if not (basis is not None and k == "basis_raw")]
        self.state = {k: np.ascontiguousarray(np.asarray(state[k], F32)) for k, _ in keys}
        for k, shape in keys:
            if self.state[k].shape != shape:
                raise ValueError(f"{k}: expected {shape}, got {self.state[k].shape}")
        self.basis_l1_scale = float(basis_l1_scale)
        self._basis = None if basis is None else np.ascontiguousarray(basis, F32)

    @property
    def base(self):
        return self.state["base_kernel"]

    @property
    def basis(self):
        if self._basis is not None:
            return self._basis
        return project_basis(self.state["basis_raw"], self.basis_l1_scale)

    def predict_coefficients(self, src):
        return controller(src, self.state)

    def __call__(self, src):
        """FoldedAEISU.forward = AEISU.forward (aeisu/model.py:546-551)."""
        return reconstruct(src, controller(src, self.state), self.base, self.basis)


def load_folded(path):
    """runtime.load_model (aeisu/runtime.py:35-56) for folded checkpoints."""
    import torch  # checkpoint container only; all arithmetic is numpy
    payload = torch.load(path, map_location="cpu", weights_only=True)
    state = payload.get("model", payload)
    scale = payload.get("basis_l1_scale", 0.5)
    return FoldedModel({k: v.numpy() for k, v in state.items()}, scale)


def pad_geometry(h, w):
    """runtime.py:79-84 replicate padding: returns (py, px, Hp, Wp)."""
    ey, ex = -h % 32, -w % 32
    py, px = 16 + ey // 2, 16 + ex // 2
    return py, px, h + 32 + ey, w + 32 + ex


def upscale(model, source, tile=128):
    """runtime.upscale (aeisu/runtime.py:70-103): [3,H,W] float -> clamped [3,2H,2W]."""
    source = np.asarray(source, F32)
    if source.ndim != 3 or source.shape[0] != 3:
        raise ValueError("Expected CHW RGB image")
    if tile < 0 or tile % 32:
        raise ValueError("tile must be zero or a positive multiple of 32")
    h, w = source.shape[-2:]
    py, px, ph, pw = pad_geometry(h, w)
    image = np.pad(source[None], ((0, 0), (0, 0), (py, ph - h - py), (px, pw - w - px)), mode="edge")
    if tile == 0:
        result = model(image)
    else:
        result = np.empty((1, 3, ph * 2, pw * 2), F32)
        for y in range(0, ph, tile):
            for x in range(0, pw, tile):
                y1, x1 = min(y + tile, ph), min(x + tile, pw)
                sy, sx = max(0, y - 32), max(0, x - 32)
                ey, ex = min(ph, y1 + 32), min(pw, x1 + 32)
                pred = model(image[:, :, sy:ey, sx:ex])
                result[:, :, 2 * y:2 * y1, 2 * x:2 * x1] = \
                    pred[:, :, 2 * (y - sy):2 * (y1 - sy), 2 * (x - sx):2 * (x1 - sx)]
    output = result[0, :, 2 * py:2 * (py + h), 2 * px:2 * (px + w)]
    if not np.isfinite(output).all():
        raise FloatingPointError("Non-finite model reconstruction")
    return np.clip(output, 0, 1).astype(F32)


def u8_to_chw(frame_hwc):
    """runtime.read_rgb (aeisu/runtime.py:17-20): uint8 HWC -> float32 CHW / 255."""
    return (np.asarray(frame_hwc).astype(F32) / F32(255)).transpose(2, 0, 1).copy()


def chw_to_u8(image):
    """runtime.save_rgb (aeisu/runtime.py:23-27): clamp, floor(x*255+0.5) -> uint8 HWC."""
    a = np.clip(np.asarray(image, F32), 0, 1).transpose(1, 2, 0)
    return np.floor(a * F32(255) + F32(0.5)).astype(np.uint8)


def upscale_u8(model, frame_hwc, tile=0):
    """uint8 HWC in, uint8 HWC 2x out, through the FP32 reference semantics."""
    return chw_to_u8(upscale(model, u8_to_chw(frame_hwc), tile))


def psnr(a, b, peak=1.0):
    d = np.asarray(a, np.float64) - np.asarray(b, np.float64)
    mse = float(np.mean(d * d))
    return float("inf") if mse == 0 else 10.0 * np.log10(peak * peak / mse)

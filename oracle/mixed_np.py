"""CPU restatement of the reduced-precision routes' arithmetic (TEST ORACLE ONLY).

Mixed FP8-E4M3/FP16 route of the reference's native runtime, quantisation point by point
(optimized/native/src/neural/srcpyr/..., paths relative to the AELabs42/AEISU checkout):

* analysis + project (SrcPyrCudaRuntime.cu:2360-2584): features rounded to f16, f16 weights,
  float accumulate, + bias, LeakyReLU, rounded to f16 -> skip
* compress (SrcPyrNativeFp8Compress.cuh:94-142, 230-236): e4m3(skip * (1/s1)); acc of e4m3
  products; acc*(s1*ws) + bias_fp8; LeakyReLU; e4m3(y * (1/s2))
* core i (SrcPyrNativeFp8Conv.cuh:414-632): grouped 3x3, zero padding; scales s[i+2] -> s[i+3]
* expand (SrcPyrNativeFp8Expand.cuh:232-305): acc*(s6*ws)+bias_fp8; LeakyReLU; e4m3(y/s7)*s7;
  pixel shuffle; + skip; rounded to f16
* refine + tail (SrcPyrNativeFp16Refine.cuh:334-557): f16 in, float accumulate, + bias,
  LeakyReLU -> f16; tail + f16(bias) -> f16 coefficients
* head (AdaptiveReconstruction.cuh:288-417): f16 coefficients, FP32 filter mix and apply.

FP16 route: the same graph with f16 weights and f16-rounded activations at every layer output.
E4M3 rounding here is an independent implementation (exponent/step arithmetic, ties to even,
saturation at +-448), cross-checked in the CPU tests against torch.float8_e4m3fn.
"""
from __future__ import annotations

import numpy as np

from . import aeisu_np as O

F32 = np.float32


def e4m3(x):
    """Round float32 values to the nearest E4M3 value (ties to even), saturating at +-448."""
    x = np.asarray(x, F32)
    a = np.minimum(np.abs(x).astype(np.float64), 448.0)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -20)))
    e = np.clip(e, -6, 8)
    step = 2.0 ** (e - 3)
    q = np.round(a / step) * step       # np.round: half to even; power-of-two steps are exact
    q = np.minimum(q, 448.0)
    return (np.sign(x) * q).astype(F32)


def f16(x):
    return np.asarray(x, F32).astype(np.float16).astype(F32)


def e4m3_decode(codes):
    c = np.asarray(codes, np.uint8)
    e = (c >> 3) & 0xF
    m = (c & 7).astype(np.float64)
    mag = np.where(e == 0, m * 2.0 ** -9, (1 + m / 8) * 2.0 ** (e.astype(np.float64) - 7))
    mag = np.where((c & 0x7F) == 0x7F, np.nan, mag)
    return np.where(c & 0x80, -mag, mag).astype(F32)


def _unshuffle(x):
    b, h, w, c = x.shape
    return x.reshape(b, h // 2, 2, w // 2, 2, c).transpose(0, 1, 3, 5, 2, 4).reshape(b, h // 2, w // 2, c * 4)


def _shuffle(x):
    b, h, w, c4 = x.shape
    c = c4 // 4
    return x.reshape(b, h, w, c, 2, 2).transpose(0, 1, 4, 2, 5, 3).reshape(b, h * 2, w * 2, c)


def _conv(x, w, b, groups=1):
    return O.conv2d_nhwc(x, w, np.zeros(w.shape[0], F32) if b is None else b, groups)


class QuantizedModel:
    """Reduced-precision restatement.  ``t`` holds SPYR8 tensors (names as in the artifact);
    ``mode`` is "mixed" (FP8 compress/core/expand) or "fp16"."""

    def __init__(self, t, mode="mixed", headroom=1.0):
        """headroom: power-of-two factor on the artifact's activation scales (1 = the
        reference's arithmetic; the B200 route uses 2 as a saturation guard)."""
        self.t, self.mode = t, mode
        self.s = (np.asarray(t["activation_scales"], F32) * F32(headroom)) if "activation_scales" in t else None
        self.basis = np.asarray(t["adaptive_basis"], F32)
        self.base = np.asarray(t["adaptive_base"], F32)
        st = np.asarray(t["analysis_stencil"], F32)
        self.stencil = {"analysis_rgb_basis": st[0:9].reshape(3, 3), "analysis_rgb_mix": st[9:12],
                        "analysis_dx_rows": st[12:15], "analysis_dy_cols": st[15:18],
                        "analysis_diag45": st[18:21], "analysis_diag135": st[21:24]}

    def w16(self, name):
        return np.asarray(self.t[f"{name}.weight_fp16"], np.float16).astype(F32)

    def _fp8_layer(self, x_q, name, s_in, groups=1):
        """acc of e4m3 products, then acc*(s_in*ws) + bias_fp8, LeakyReLU."""
        w = e4m3_decode(self.t[f"{name}.weight_fp8"])
        acc = _conv(x_q, w, None, groups)
        scale = (F32(s_in) * np.asarray(self.t[f"{name}.weight_scale"], F32)).astype(F32)
        return O.leaky((acc * scale + np.asarray(self.t[f"{name}.bias_fp8"], F32)).astype(F32))

    def _f16_layer(self, x, name, act=True, groups=1, bias=None):
        y = _conv(x, self.w16(name), np.asarray(self.t[f"{name}.bias"], F32) if bias is None else bias, groups)
        return O.leaky(y) if act else y

    def predict_coefficients(self, src):
        s, t = self.s, self.t
        feat = np.ascontiguousarray(O.feature8(src, self.stencil).transpose(0, 2, 3, 1))
        skip = f16(self._f16_layer(f16(_unshuffle(feat)), "project"))
        if self.mode == "mixed":
            q = e4m3(_unshuffle(skip) * (F32(1) / s[1]))
            low = e4m3(self._fp8_layer(q, "compress", s[1]) * (F32(1) / s[2]))
            for i in range(4):
                low = e4m3(self._fp8_layer(low, f"bottleneck{i}", s[i + 2], groups=2) * (F32(1) / s[i + 3]))
            up = e4m3(self._fp8_layer(low, "expand", s[6]) * (F32(1) / s[7])) * s[7]
        else:
            low = f16(self._f16_layer(_unshuffle(skip), "compress"))
            for i in range(4):
                low = f16(self._f16_layer(low, f"bottleneck{i}", groups=2))
            up = self._f16_layer(low, "expand")
        dec = f16(_shuffle(up) + skip)
        ref = f16(self._f16_layer(dec, "refine"))
        meta = f16(self._f16_layer(ref, "tail", act=False, bias=f16(np.asarray(t["tail.bias"], F32))))
        return np.ascontiguousarray(meta.transpose(0, 3, 1, 2))

    def __call__(self, src):
        return O.reconstruct(src, self.predict_coefficients(src), self.base, self.basis)


def upscale(model, source, tile=0):
    """runtime.upscale semantics (aeisu/runtime.py:70-103) with a QuantizedModel."""
    return O.upscale(model, source, tile)

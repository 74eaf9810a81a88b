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

INT8 route of the conventional-CUDA deployment (optimized/shader/runtime.py:173-221 over
optimized/shader/src/int8_kernels.cuh), from the shader_precision_v1 record:

* int8 code q(x) = clamp(round_half_even(x), -127, 127) (quantize_s8, int8_kernels.cuh:2-4)
* compress (int8_body COMPRESS, :18-31, 46-52): q(skip * (1/s1)); integer dot products with the
  int8 weights; acc*factor + bias in one rounding; LeakyReLU; q(y * (1/s2))
* bottleneck 0..3 (int8_pair, :159-199, grouped 3x3, zero padding): outputs q(y * (1/s3..s6))
* expand (int8_body EXPAND, :46-59): q(y * (1/s7)); code*s7 + skip in one rounding; f16
* project, refine, tail and head as in this module's f16 layers (float accumulation; the
  reference's own FP16 kernels accumulate some sums in half, fusion_kernels.cu:174-184), with the
  tail adding its FP32 bias.

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


def int8_code(x):
    """quantize_s8 of an already scaled float32 value: round half to even, clamp to +-127."""
    return np.clip(np.rint(np.asarray(x, F32)), -127, 127).astype(F32)


def _fma(a, b, c):
    """float32 a*b + c with one rounding (the products here are exact in float64)."""
    return (np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64)).astype(F32)


INT8_LAYERS = ("compress", "bottleneck0", "bottleneck1", "bottleneck2", "bottleneck3", "expand")


def int8_record_tensors(record):
    """The tensors of a shader_precision_v1 record under this module's names."""
    a = lambda v, dt=F32: np.asarray(v).astype(dt)
    t = {"activation_scales": a(record["activation_scales"]), "adaptive_basis": a(record["bank"]),
         "adaptive_base": a(record["base"]), "analysis_stencil": a(record["analysis_parameters"])}
    for name in ("project", "refine", "tail"):
        t[f"{name}.weight_fp16"] = a(record["half_weights"][name], np.float16)
        t[f"{name}.bias"] = a(record["half_biases"][name])
    for name in INT8_LAYERS:
        t[f"{name}.weight_int8"] = a(record["int8_weights"][name], np.int8)
        t[f"{name}.factor"] = a(record["int8_factors"][name])
        t[f"{name}.bias_int8"] = a(record["int8_biases"][name])
    return t


def _unshuffle(x):
    b, h, w, c = x.shape
    return x.reshape(b, h // 2, 2, w // 2, 2, c).transpose(0, 1, 3, 5, 2, 4).reshape(b, h // 2, w // 2, c * 4)


def _shuffle(x):
    b, h, w, c4 = x.shape
    c = c4 // 4
    return x.reshape(b, h, w, c, 2, 2).transpose(0, 1, 4, 2, 5, 3).reshape(b, h * 2, w * 2, c)


def _conv(x, w, b, groups=1):
    return O.conv2d_nhwc(x, w, np.zeros(w.shape[0], F32) if b is None else b, groups)


def own_weights_state(t, state16):
    """FP32 folded state that holds the mixed route's own weights: the FP8 layers (compress_270,
    the four bottleneck layers, expand_270) as their E4M3 codes times the per-output-channel
    weight_scale, with bias_fp8, the layers the mixed route runs in FP16 (project_540,
    refine_540, metadata_head) as stored.  ``state16`` is spyr8.folded_state_from_spyr8(t)[0];
    the mixed route's _fp8_layer applies exactly these weights to its quantised activations."""
    st = dict(state16)

    def deq(name):
        w = e4m3_decode(t[f"{name}.weight_fp8"]).astype(F32)
        ws = np.asarray(t[f"{name}.weight_scale"], F32).reshape(-1, *([1] * (w.ndim - 1)))
        return (w * ws).astype(F32), np.asarray(t[f"{name}.bias_fp8"], F32)

    for name, key in (("compress", "compress_270"), ("expand", "expand_270")):
        st[f"{key}.weight"], st[f"{key}.bias"] = deq(name)
    for i in range(4):
        w, b = deq(f"bottleneck{i}")
        st[f"bottleneck_270_a{i + 1}.weight"], st[f"bottleneck_270_b{i + 1}.weight"] = w[:32], w[32:]
        st[f"bottleneck_270_a{i + 1}.bias"], st[f"bottleneck_270_b{i + 1}.bias"] = b[:32], b[32:]
    return st


class QuantizedModel:
    """Reduced-precision restatement.  ``t`` holds SPYR8 tensors (names as in the artifact) for
    ``mode`` "mixed" (FP8 compress/core/expand) or "fp16", or the tensors of
    ``int8_record_tensors`` for ``mode`` "int8"."""

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

    def _int8_layer(self, codes, name, groups=1):
        """Integer dot products (exact in float32: |sum| < 2^24), acc*factor + bias, LeakyReLU."""
        acc = _conv(codes, np.asarray(self.t[f"{name}.weight_int8"], F32), None, groups)
        return O.leaky(_fma(acc, self.t[f"{name}.factor"], self.t[f"{name}.bias_int8"]))

    def _f16_layer(self, x, name, act=True, groups=1, bias=None):
        y = _conv(x, self.w16(name), np.asarray(self.t[f"{name}.bias"], F32) if bias is None else bias, groups)
        return O.leaky(y) if act else y

    def predict_coefficients(self, src):
        s, t = self.s, self.t
        feat = np.ascontiguousarray(O.feature8(src, self.stencil).transpose(0, 2, 3, 1))
        skip = f16(self._f16_layer(f16(_unshuffle(feat)), "project"))
        if self.mode == "int8":
            inv = lambda i: F32(1) / s[i]
            low = int8_code(self._int8_layer(int8_code(_unshuffle(skip) * inv(1)), "compress") * inv(2))
            for i in range(4):
                low = int8_code(self._int8_layer(low, f"bottleneck{i}", groups=2) * inv(i + 3))
            q7 = int8_code(self._int8_layer(low, "expand") * inv(7))
            dec = f16(_fma(_shuffle(q7), s[7], skip))
        elif self.mode == "mixed":
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
        if self.mode != "int8":
            dec = f16(_shuffle(up) + skip)
        ref = f16(self._f16_layer(dec, "refine"))
        tail_bias = np.asarray(t["tail.bias"], F32)
        meta = f16(self._f16_layer(ref, "tail", act=False, bias=tail_bias if self.mode == "int8" else f16(tail_bias)))
        return np.ascontiguousarray(meta.transpose(0, 3, 1, 2))

    def __call__(self, src):
        return O.reconstruct(src, self.predict_coefficients(src), self.base, self.basis)


def upscale(model, source, tile=0):
    """runtime.upscale semantics (aeisu/runtime.py:70-103) with a QuantizedModel."""
    return O.upscale(model, source, tile)

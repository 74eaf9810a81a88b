"""Python operator API over the C ABI, mirroring the reference's aeisu.runtime.

Reference surface mirrored (paths relative to the AELabs42/AEISU checkout):

* ``load_model(path, device)``  -> aeisu/runtime.py:45-56 (folded ``.pt`` and training
  checkpoints, folded on load by ``aeisu_b200.fold``); also SPYR8 ``.bin``
  and the INT8/FP16 ``shader_precision_v1`` ``.pt`` (optimized/shader/runtime.py:37-59)
* ``upscale(model, source, tile=128)`` -> aeisu/runtime.py:70-103 (same padding, tiling,
  ValueError / FloatingPointError behaviour, clamped CHW float32 result)
* ``model(src)`` / ``model.predict_coefficients(src)`` -> FoldedAEISU.forward /
  predict_coefficients (aeisu/model.py:494-551)
* ``read_rgb`` / ``save_rgb`` -> aeisu/runtime.py:17-27

plus the deployment entry point ``upscale_u8`` (uint8 HWC frames in and out, batched).
Arrays may be numpy arrays, CPU tensors (host I/O through the library's copies) or CUDA
tensors on the model's device (device I/O on the current torch stream).  All compute runs
in ``libaeisu_b200.so``; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

from . import _lib, fold

# FoldedAEISU.state_dict() order and shapes (aeisu/model.py:554-583).
_CONVS = (
    ("project_540", 32, 32, 1),
    ("compress_270", 128, 64, 1),
    *((f"bottleneck_270_{b}{i}", 32, 32, 3) for b in ("a", "b") for i in range(1, 5)),
    ("expand_270", 64, 128, 1),
    ("refine_540", 32, 64, 3),
    ("metadata_head", 64, 64, 1),
)
FOLDED_KEYS = (
    ("analysis_rgb_basis", (3, 3)), ("analysis_rgb_mix", (3,)), ("analysis_dx_rows", (3,)),
    ("analysis_dy_cols", (3,)), ("analysis_diag45", (3,)), ("analysis_diag135", (3,)),
    ("base_kernel", (25, 4)), ("basis_raw", (16, 4, 25)),
    *(item for name, cin, cout, k in _CONVS
      for item in ((f"{name}.weight", (cout, cin, k, k)), (f"{name}.bias", (cout,)))),
)
SPYR8_MAGIC = b"SPYR8F8\0"
CUDA_STREAM_LEGACY = 0x1   # cudaStreamLegacy of cuda_runtime_api.h
# optimized/shader/runtime.py:34, 41-43: the one published INT8/FP16 policy
INT8_LAYERS = ("compress", "bottleneck0", "bottleneck1", "bottleneck2", "bottleneck3", "expand")
INT8_POLICY = {"project": "fp16", **{name: "int8" for name in INT8_LAYERS}, "refine": "fp16", "tail": "fp16"}


def int8_arrays(record):
    """The arrays of a shader_precision_v1 record (optimized/shader/weights/aeisu_int8_fp16.pt),
    checked as MixedRuntime.__init__ checks them (optimized/shader/runtime.py:37-43), as
    contiguous numpy arrays keyed by their aeisu_int8_artifact field."""
    if not isinstance(record, dict) or record.get("format") != "shader_precision_v1" \
            or record.get("precision_policy") != INT8_POLICY or record.get("all_int8"):
        raise ValueError("This runner accepts only the published mixed INT8/FP16 policy")

    def arr(value, dtype, shape):
        a = np.ascontiguousarray(np.asarray(value.numpy() if hasattr(value, "numpy") else value).astype(dtype))
        if a.shape != shape:
            raise ValueError(f"INT8 artifact tensor has shape {a.shape}, expected {shape}")
        return a

    half, hb = record["half_weights"], record["half_biases"]
    out = {"analysis": arr(record["analysis_parameters"], np.float32, (24,)),
           "base": arr(record["base"], np.float32, (25, 4)),
           "bank": arr(record["bank"], np.float32, (25, 16, 4)),
           "project_w": arr(half["project"], np.float16, (32, 32, 1, 1)).view(np.uint16),
           "refine_w": arr(half["refine"], np.float16, (64, 32, 3, 3)).view(np.uint16),
           "tail_w": arr(half["tail"], np.float16, (64, 64, 1, 1)).view(np.uint16),
           "project_b": arr(hb["project"], np.float32, (32,)),
           "refine_b": arr(hb["refine"], np.float32, (64,)),
           "tail_b": arr(hb["tail"], np.float32, (64,)),
           "activation_scales": arr(record["activation_scales"], np.float32, (10,))}
    shapes = {"compress": (64, 128, 1, 1), "expand": (128, 64, 1, 1)}
    for name in INT8_LAYERS:
        co = shapes.get(name, (64, 32, 3, 3))
        out[f"{name}.w"] = arr(record["int8_weights"][name], np.int8, co)
        out[f"{name}.factor"] = arr(record["int8_factors"][name], np.float32, (co[0],))
        out[f"{name}.bias"] = arr(record["int8_biases"][name], np.float32, (co[0],))
    return out


def _device_index(device) -> int:
    if isinstance(device, int):
        return device
    text = str(device)
    if text in ("cuda", "auto"):
        return 0
    if text.startswith("cuda:"):
        return int(text.split(":", 1)[1])
    raise ValueError(f"aeisu_b200 runs on CUDA devices only, got device={device!r}")


def flatten_folded(state) -> np.ndarray:
    """Concatenate a folded state dict (tensors or arrays) in FoldedAEISU.state_dict() order."""
    parts = []
    for key, shape in FOLDED_KEYS:
        if key not in state:
            raise ValueError(f"Checkpoint is missing {key}")
        value = state[key]
        value = value.detach().cpu().numpy() if hasattr(value, "detach") else np.asarray(value)
        if tuple(value.shape) != shape:
            raise ValueError(f"{key}: expected shape {shape}, got {tuple(value.shape)}")
        parts.append(np.ascontiguousarray(value, np.float32).reshape(-1))
    extra = set(state) - {k for k, _ in FOLDED_KEYS}
    if extra:
        raise ValueError(f"Unexpected checkpoint keys: {sorted(extra)[:4]}")
    flat = np.concatenate(parts)
    assert flat.size == _lib.FOLDED_VALUES
    return flat


def _checkpoint_state(payload):
    """runtime.checkpoint_state (aeisu/runtime.py:35-42)."""
    if isinstance(payload, dict):
        for key in ("model", "model_state_dict", "state_dict"):
            if isinstance(payload.get(key), dict):
                return payload[key]
        if payload and all(hasattr(v, "shape") for v in payload.values()):
            return payload
    raise ValueError("Checkpoint does not contain a tensor state dictionary")


class _Array:
    """A view of a caller array as (pointer, is_device, keepalive, torch-ness)."""

    def __init__(self, value, dtype, device_index):
        self.torch = None
        self.value = value
        try:
            import torch
        except ImportError:  # numpy-only callers
            torch = None
        if torch is not None and isinstance(value, torch.Tensor):
            self.torch = torch
            want = {np.float32: torch.float32, np.uint8: torch.uint8}[dtype]
            if value.is_cuda:
                if value.device.index != device_index:
                    raise ValueError(f"tensor is on {value.device}, model on cuda:{device_index}")
                self.keep = value.to(want).contiguous()
                self.ptr = self.keep.data_ptr()
                self.device = True
                # torch's default stream reports handle 0, which the C ABI reads as "the model's
                # own stream" (non-blocking: unordered with the caller's work); name the legacy
                # default stream explicitly instead (cudaStreamLegacy)
                self.stream = torch.cuda.current_stream(value.device).cuda_stream or CUDA_STREAM_LEGACY
                return
            self.keep = value.detach().to(want).contiguous().numpy()
        else:
            self.keep = np.ascontiguousarray(value, dtype)
        self.ptr = self.keep.ctypes.data
        self.device = False
        self.stream = None


class Model:
    """A model resident on one GPU (one C-ABI handle)."""

    def __init__(self, handle, device_index, precision, basis_l1_scale=0.5):
        self._h = handle
        self.device_index = device_index
        self.precision = precision
        self.basis_l1_scale = basis_l1_scale

    # -- construction ----------------------------------------------------------------
    @classmethod
    def from_folded_state(cls, state, device="cuda", precision="fp32", basis_l1_scale=0.5):
        flat = flatten_folded(state)
        dev = _device_index(device)
        h = C.c_void_p()
        _lib.check(_lib.lib().aeisu_open_folded(flat.ctypes.data, flat.size, float(basis_l1_scale),
                                                _lib.PRECISIONS[precision], dev, C.byref(h)))
        return cls(h, dev, precision, basis_l1_scale)

    @classmethod
    def from_spyr8_bytes(cls, data: bytes, device="cuda", precision="mixed", activation_headroom=1.0):
        """A SPYR8 artifact image.  activation_headroom (a power of two, mixed route only)
        multiplies the artifact's FP8 activation scales; 1 runs its own quantisation points."""
        dev = _device_index(device)
        buf = C.create_string_buffer(data, len(data))
        h = C.c_void_p()
        _lib.check(_lib.lib().aeisu_open_spyr8_headroom(buf, len(data), _lib.PRECISIONS[precision], dev,
                                                        float(activation_headroom), C.byref(h)))
        return cls(h, dev, precision)

    @classmethod
    def from_int8_record(cls, record, device="cuda"):
        """The INT8/FP16 route of a shader_precision_v1 record (precision "int8" only)."""
        a = int8_arrays(record)
        dev = _device_index(device)
        st = _lib.Int8Artifact()
        for key in ("analysis", "base", "bank", "project_w", "refine_w", "tail_w", "project_b", "refine_b",
                    "tail_b", "activation_scales"):
            setattr(st, key, a[key].ctypes.data)
        for i, name in enumerate(INT8_LAYERS):
            st.int8_w[i] = a[f"{name}.w"].ctypes.data
            st.int8_factor[i] = a[f"{name}.factor"].ctypes.data
            st.int8_bias[i] = a[f"{name}.bias"].ctypes.data
        h = C.c_void_p()
        _lib.check(_lib.lib().aeisu_open_int8(C.byref(st), dev, C.byref(h)))
        return cls(h, dev, "int8")

    def sibling(self):
        """Another handle on the same model and GPU sharing this one's device weights, with its
        own stream and workspace (aeisu_open_sibling; CudaRuntime::CreateSibling,
        SrcPyrCudaRuntime.cu:5392-5402): one handle per host thread, one weight copy."""
        h = C.c_void_p()
        _lib.check(_lib.lib().aeisu_open_sibling(self._handle(), C.byref(h)))
        return type(self)(h, self.device_index, self.precision, self.basis_l1_scale)

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().aeisu_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _handle(self):
        if not self._h:
            raise ValueError("model is closed")
        return self._h

    # -- introspection ---------------------------------------------------------------
    @property
    def report(self) -> str:
        return _lib.lib().aeisu_report(self._handle()).decode()

    @property
    def device_bytes(self) -> int:
        return int(_lib.lib().aeisu_device_bytes(self._handle()))

    @property
    def kernel_launches(self) -> int:
        return int(_lib.lib().aeisu_kernel_launches(self._handle()))

    def timings(self) -> dict:
        t = _lib.Timings()
        _lib.check(_lib.lib().aeisu_timings_get(self._handle(), C.byref(t)))
        return {name: getattr(t, name) for name, _ in t._fields_}

    def set_detailed_timing(self, on: bool):
        _lib.check(_lib.lib().aeisu_set_detailed_timing(self._handle(), int(bool(on))))

    def set_timeout(self, ms: float):
        _lib.check(_lib.lib().aeisu_set_timeout(self._handle(), float(ms)))

    def set_fused_head(self, on: bool):
        """Tensor-core routes: reconstruct in a separate head kernel over coefficients kept in
        device memory (default) or inside the controller's last kernel, so that they never reach
        device memory; the output is the same bit for bit."""
        _lib.check(_lib.lib().aeisu_set_fused_head(self._handle(), int(bool(on))))

    def set_workspace_limit(self, nbytes: int):
        """Bound the intermediate-tensor bytes of one call; larger batches run in passes."""
        _lib.check(_lib.lib().aeisu_set_workspace_limit(self._handle(), int(nbytes)))

    def synchronize(self, stream=None, timeout_ms=60000.0):
        _lib.check(_lib.lib().aeisu_synchronize(self._handle(), stream, float(timeout_ms)))

    # -- reference operator surface ----------------------------------------------------
    def _out(self, arr: _Array, shape, dtype):
        if arr.device:
            t = arr.torch
            return t.empty(shape, dtype={np.float32: t.float32, np.uint8: t.uint8}[dtype],
                           device=f"cuda:{self.device_index}")
        return np.empty(shape, dtype)

    @staticmethod
    def _ptr(out):
        return out.data_ptr() if hasattr(out, "data_ptr") else out.ctypes.data

    def _wrap(self, arr: _Array, out):
        if arr.torch is not None and not arr.device and isinstance(out, np.ndarray):
            return arr.torch.from_numpy(out)
        return out

    def predict_coefficients(self, source):
        """Metadata [B,64,H/2,W/2] (NCHW, as FoldedAEISU.predict_coefficients returns)."""
        a = _Array(source, np.float32, self.device_index)
        if a.keep.ndim != 4 or a.keep.shape[1] != 3:
            raise ValueError(f"Expected source RGB [B,3,H,W], got {tuple(a.keep.shape)}")
        b, _, h, w = a.keep.shape
        out = self._out(a, (b, h // 2, w // 2, 64), np.float32)
        _lib.check(_lib.lib().aeisu_predict_coefficients(
            self._handle(), a.ptr, b, h, w, self._ptr(out), _lib.IO_DEVICE if a.device else _lib.IO_HOST,
            a.stream))
        out = out.permute(0, 3, 1, 2) if a.device else out.transpose(0, 3, 1, 2)
        return self._wrap(a, out)

    def activation_stats(self, frames):
        """Calibration statistics of this FP32 model over uint8 frames [n,H,W,3] or [H,W,3]:
        (peaks[10], means[448]) as aeisu_activation_stats defines them."""
        a = _Array(frames, np.uint8, self.device_index)
        x = a.keep
        if x.ndim == 3:
            x = x[None]
        if x.ndim != 4 or x.shape[-1] != 3:
            raise ValueError(f"Expected uint8 frames [n,H,W,3], got {tuple(x.shape)}")
        peaks = np.zeros(10, np.float32)
        means = np.zeros(448, np.float32)
        _lib.check(_lib.lib().aeisu_activation_stats(
            self._handle(), a.ptr, x.shape[0], x.shape[1], x.shape[2], _lib.IO_DEVICE if a.device else _lib.IO_HOST,
            peaks.ctypes.data, means.ctypes.data, a.stream))
        return peaks, means

    def __call__(self, source):
        """FoldedAEISU.forward: unclipped 2x RGB [B,3,2H,2W] of a padded batch."""
        a = _Array(source, np.float32, self.device_index)
        if a.keep.ndim != 4 or a.keep.shape[1] != 3:
            raise ValueError(f"Expected source RGB [B,3,H,W], got {tuple(a.keep.shape)}")
        b, _, h, w = a.keep.shape
        out = self._out(a, (b, 3, 2 * h, 2 * w), np.float32)
        _lib.check(_lib.lib().aeisu_forward_f32(
            self._handle(), a.ptr, b, h, w, self._ptr(out), _lib.IO_DEVICE if a.device else _lib.IO_HOST,
            a.stream))
        return self._wrap(a, out)

    forward = __call__

    def upscale_f32(self, source, tile=128):
        """Unclipped upscale of one CHW or a batch of NCHW float frames."""
        a = _Array(source, np.float32, self.device_index)
        x = a.keep
        single = x.ndim == 3
        if x.ndim not in (3, 4) or x.shape[-3] != 3:
            raise ValueError("Expected CHW RGB image")
        n = 1 if single else x.shape[0]
        h, w = x.shape[-2:]
        out = self._out(a, (n, 3, 2 * h, 2 * w), np.float32)
        _lib.check(_lib.lib().aeisu_upscale_f32(
            self._handle(), a.ptr, n, h, w, int(tile), self._ptr(out),
            _lib.IO_DEVICE if a.device else _lib.IO_HOST, a.stream))
        out = out[0] if single else out
        return self._wrap(a, out)

    def upscale_u8(self, frames, tile=0, out=None):
        """uint8 HWC (or NHWC) frames -> uint8 2x frames; clamp + floor(x*255+0.5)."""
        a = _Array(frames, np.uint8, self.device_index)
        x = a.keep
        single = x.ndim == 3
        if x.ndim not in (3, 4) or x.shape[-1] != 3:
            raise ValueError("Expected HWC RGB uint8 frames")
        n = 1 if single else x.shape[0]
        h, w = x.shape[-3:-1]
        shape = (2 * h, 2 * w, 3) if single else (n, 2 * h, 2 * w, 3)
        if out is None:
            out = self._out(a, shape, np.uint8)
        elif tuple(out.shape) != shape:
            raise ValueError(f"out must have shape {shape}")
        _lib.check(_lib.lib().aeisu_upscale_u8(
            self._handle(), a.ptr, n, h, w, int(tile), self._ptr(out),
            _lib.IO_DEVICE if a.device else _lib.IO_HOST, a.stream))
        return self._wrap(a, out)

    def upscale_u8_band(self, frame, band, bands, out=None):
        """Row band `band` of `bands` of one uint8 HWC frame (aeisu_upscale_u8_band): writes that
        band's output rows of the 2x frame into `out` (allocated, zero-filled, when None) and
        returns it.  The bands of 0..bands-1 together give exactly upscale_u8(frame, 0)."""
        a = _Array(frame, np.uint8, self.device_index)
        x = a.keep
        if x.ndim != 3 or x.shape[-1] != 3:
            raise ValueError("Expected one HWC RGB uint8 frame")
        h, w = x.shape[:2]
        shape = (2 * h, 2 * w, 3)
        if out is None:
            out = self._out(a, shape, np.uint8)
            out[...] = 0
        elif tuple(out.shape) != shape:
            raise ValueError(f"out must have shape {shape}")
        _lib.check(_lib.lib().aeisu_upscale_u8_band(
            self._handle(), a.ptr, h, w, int(band), int(bands), self._ptr(out),
            _lib.IO_DEVICE if a.device else _lib.IO_HOST, a.stream))
        return self._wrap(a, out)


def load_model(path, device="cuda", precision=None, activation_headroom=1.0) -> Model:
    """runtime.load_model (aeisu/runtime.py:45-56) for folded ``.pt`` checkpoints, plus
    SPYR8 ``.bin`` artifacts and the INT8/FP16 ``shader_precision_v1`` ``.pt``
    (optimized/shader/runtime.py:37-59).  precision defaults to fp32 for a folded ``.pt``,
    mixed for SPYR8 and int8 (its only precision) for the INT8 artifact.  activation_headroom:
    the power of two the mixed route multiplies a SPYR8 artifact's activation scales by (1, the
    default, runs the artifact's own quantisation points)."""
    path = Path(path)
    with path.open("rb") as f:
        head = f.read(8)
    if head == SPYR8_MAGIC:
        return Model.from_spyr8_bytes(path.read_bytes(), device, precision or "mixed", activation_headroom)
    import torch  # checkpoint container only
    payload = torch.load(path, map_location="cpu", weights_only=True)
    if isinstance(payload, dict) and payload.get("format") == "shader_precision_v1":
        if precision not in (None, "int8"):
            raise ValueError("the INT8/FP16 artifact runs only at precision int8")
        return Model.from_int8_record(payload, device)
    state = _checkpoint_state(payload)
    scale = payload.get("basis_l1_scale", payload.get("config", {}).get("basis_l1_scale", 0.5)) \
        if isinstance(payload, dict) else 0.5
    if fold.is_training_state(state):
        # a train.py checkpoint: fold its training-only branches as load_model does
        # (aeisu/runtime.py:49-52, fold_model of aeisu/model.py:599-602)
        state = fold.fold_training_state(state)
    return Model.from_folded_state(state, device, precision or "fp32", scale)


def upscale(model: Model, source, tile: int = 128):
    """runtime.upscale (aeisu/runtime.py:70-103): CHW float [0,1] -> clamped CHW 2x float."""
    shape = tuple(source.shape)
    if len(shape) != 3 or shape[0] != 3:
        raise ValueError("Expected CHW RGB image")
    if tile < 0 or tile % 32:
        raise ValueError("tile must be zero or a positive multiple of 32")
    out = model.upscale_f32(source, tile)
    if hasattr(out, "isfinite"):
        if not bool(out.isfinite().all()):
            raise FloatingPointError("Non-finite model reconstruction")
        return out.clamp(0, 1)
    if not np.isfinite(out).all():
        raise FloatingPointError("Non-finite model reconstruction")
    return np.clip(out, 0, 1)


def upscale_u8(model: Model, frames, tile: int = 0, out=None):
    return model.upscale_u8(frames, tile, out)


def read_rgb(path):
    """runtime.read_rgb (aeisu/runtime.py:17-20): image file -> float32 CHW in [0,1] (torch)."""
    import torch
    from PIL import Image
    with Image.open(path) as image:
        array = np.array(image.convert("RGB"), dtype=np.uint8, copy=True)
    return torch.from_numpy(array).permute(2, 0, 1).float().div(255)


def save_rgb(path, image):
    """runtime.save_rgb (aeisu/runtime.py:23-27): clamp, floor(x*255+0.5), PNG."""
    from PIL import Image
    a = image.detach().cpu().clamp(0, 1).permute(1, 2, 0).numpy() if hasattr(image, "detach") \
        else np.clip(np.asarray(image, np.float32), 0, 1).transpose(1, 2, 0)
    a = np.floor(a * 255 + 0.5).astype(np.uint8)
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    Image.fromarray(a).save(path)

"""Encoded-Y PSNR / SSIM on the GPU: ``distortion()`` of aeisu/metrics.py:17-39 over the C ABI's
``aeisu_distortion`` (one FP64 CUDA pass over both images; there is no CPU fallback).

``distortion(prediction, target, crop=2)`` takes the same float CHW RGB images as the reference
(the prediction as ``upscale`` returns it, the target as ``read_rgb`` gives it) and returns the
same dictionary ``{"y_mse", "y_psnr", "y_ssim"}``, raising ``ValueError`` where the reference does.
CUDA tensors are read where they are (device I/O on their own stream); numpy arrays and CPU
tensors are copied to ``device``.  ``distortion_batch`` scores n pairs in one call.  The
arithmetic is float32 input, FP64 metric: inputs must be float32 (or float16 / bfloat16, which
float32 holds exactly); float64 inputs are refused rather than rounded.
"""
from __future__ import annotations

import math

import numpy as np

from . import _lib
from .runtime import _Array, _device_index

_SIZE = "Prediction and target must be same-size CHW RGB"


def luma(rgb):
    """metrics.py:11-14: BT.601 encoded luma of a float CHW image, keeping the channel axis."""
    weights = rgb.new_tensor([65.481, 128.553, 24.966]).reshape(3, 1, 1)
    return ((rgb * weights).sum(dim=0, keepdim=True) + 16) / 255


def _dtype_ok(x):
    name = str(getattr(x, "dtype", ""))
    return name.replace("torch.", "") in ("float32", "float16", "bfloat16")


def _scores(v):
    mse, psnr, ssim = (float(x) for x in v)
    return {"y_mse": mse, "y_psnr": math.inf if mse == 0 else psnr, "y_ssim": ssim}


def _run(prediction, target, batched, crop, device):
    for x in (prediction, target):
        if not _dtype_ok(x):
            raise TypeError(f"distortion expects float32 images, got {getattr(x, 'dtype', type(x))}")
    if tuple(prediction.shape) != tuple(target.shape) or prediction.ndim != 3 + batched:
        raise ValueError(_SIZE)
    if prediction.shape[-3] != 3:
        raise ValueError(_SIZE)
    on_gpu = [bool(getattr(x, "is_cuda", False)) for x in (prediction, target)]
    if on_gpu[0] != on_gpu[1]:
        raise ValueError("prediction and target must both be CUDA tensors or both host arrays")
    if on_gpu[0]:
        if prediction.device != target.device:
            raise ValueError("prediction and target are on different devices")
        dev = prediction.device.index
    else:
        dev = _device_index(device)
    a = _Array(prediction, np.float32, dev)
    b = _Array(target, np.float32, dev)
    n = prediction.shape[0] if batched else 1
    h, w = prediction.shape[-2:]
    out = np.zeros((n, 3), np.float64)
    status = _lib.lib().aeisu_distortion(a.ptr, b.ptr, n, h, w, int(crop),
                                         _lib.IO_DEVICE if a.device else _lib.IO_HOST, dev,
                                         out.ctypes.data, a.stream)
    if status == _lib.NONFINITE:
        raise ValueError("Prediction and target must be finite")
    _lib.check(status)
    return out


def distortion(prediction, target, crop=2, device="cuda"):
    """aeisu/metrics.py:17-39: {"y_mse", "y_psnr", "y_ssim"} of one CHW pair, computed on the GPU."""
    return _scores(_run(prediction, target, False, crop, device)[0])


def distortion_batch(predictions, targets, crop=2, device="cuda"):
    """distortion() of n pairs given as [n, 3, H, W]: one dictionary per pair, one GPU call.
    A non-finite value in any pair raises ValueError for the batch."""
    return [_scores(v) for v in _run(predictions, targets, True, crop, device)]

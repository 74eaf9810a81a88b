"""Drop-in ``reconstruct`` for training: aeisu/reconstruction.py:29-83 on the GPU, with its backward.

``reconstruct(source, metadata, base, basis, *, trim=0, gradient_stride=1, phase=0)`` takes the
reference's arguments and returns the same unclipped 2x RGB of the core.  It is a
``torch.autograd.Function`` over the C ABI (``aeisu_reconstruct_f32`` forward,
``aeisu_reconstruct_backward_f32`` backward), so ``loss.backward()`` in a training loop such as
train.py:99-103 gives the reference's gradients: dense metadata gradients through the
coefficient clamp, and base/basis gradients summed over every core pixel (stride 1), over the
phase-selected pixels weighted stride**2 (stride > 1), or none at all (stride 0, as the reference
leaves ``.grad`` unset).

The arithmetic is float32, as the reference's default: inputs may be float32, float16 or
bfloat16 (``metadata`` from a bf16-autocast controller is cast to float32 as the reference's
``metadata.to(dtype)`` does, and its gradient flows back in its own dtype); float64 is refused
rather than computed at a lower precision.  All tensors must be CUDA tensors on one device; there
is no CPU fallback.  Gradients with respect to ``source`` are not computed (training sources are
data): a source that requires grad is refused.  Errors follow the reference: ``ValueError`` with
its messages for bad geometry, trim, stride or phase.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

_FLOATS = (torch.float32, torch.float16, torch.bfloat16)


def _check(source, metadata, trim, gradient_stride, phase):
    """reconstruction.py:37-52, in the reference's order and words."""
    if source.ndim != 4 or source.shape[1] != 3:
        raise ValueError("Expected NCHW RGB source")
    if trim < 0 or trim % 2 or (trim and trim < 4):
        raise ValueError("trim must be zero or an even HR border of at least 4 pixels")
    if gradient_stride < 0 or phase < 0:
        raise ValueError("gradient_stride and phase must be nonnegative")
    b, _, h, w = source.shape
    off = trim // 2
    ch, cw = h - 2 * off, w - 2 * off
    if ch <= 0 or cw <= 0 or tuple(metadata.shape) != (b, 64, h // 2, w // 2) or h % 2 or w % 2:
        raise ValueError("Source, metadata or trim geometry is invalid")
    return b, h, w, ch, cw


def _stream(device):
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


class _Reconstruct(torch.autograd.Function):
    @staticmethod
    def forward(ctx, source, metadata, base, basis, trim, gradient_stride, phase):
        b, h, w, ch, cw = _check(source, metadata, trim, gradient_stride, phase)
        dev = source.device
        out = torch.empty((b, 3, 2 * ch, 2 * cw), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(_lib.lib().aeisu_reconstruct_f32(
                source.data_ptr(), metadata.data_ptr(), base.data_ptr(), basis.data_ptr(), b, h, w, trim,
                dev.index, out.data_ptr(), _stream(dev)))
        ctx.save_for_backward(source, metadata, basis)
        ctx.geom = (b, h, w, trim, gradient_stride, phase)
        return out

    @staticmethod
    def backward(ctx, grad):
        source, metadata, basis = ctx.saved_tensors
        b, h, w, trim, stride, phase = ctx.geom
        dev = source.device
        grad = grad.to(torch.float32).contiguous()
        gmeta = torch.empty_like(metadata)
        want = stride > 0 and (ctx.needs_input_grad[2] or ctx.needs_input_grad[3])
        gbase = torch.empty((25, 4), dtype=torch.float32, device=dev) if want else None
        gbasis = torch.empty((25, 16, 4), dtype=torch.float32, device=dev) if want else None
        with torch.cuda.device(dev):
            _lib.check(_lib.lib().aeisu_reconstruct_backward_f32(
                source.data_ptr(), metadata.data_ptr(), basis.data_ptr(), grad.data_ptr(), b, h, w, trim,
                stride if want else 0, phase, dev.index, gmeta.data_ptr(),
                gbase.data_ptr() if want else None, gbasis.data_ptr() if want else None, _stream(dev)))
        return (None, gmeta if ctx.needs_input_grad[1] else None,
                gbase if want and ctx.needs_input_grad[2] else None,
                gbasis if want and ctx.needs_input_grad[3] else None, None, None, None)


def reconstruct(source, metadata, base, basis, *, trim=0, gradient_stride=1, phase=0):
    """aeisu.reconstruction.reconstruct on the GPU: unclipped 2x RGB [B, 3, 2(H - trim), 2(W - trim)]."""
    if source.ndim != 4 or source.shape[1] != 3:
        raise ValueError("Expected NCHW RGB source")
    tensors = (source, metadata, base, basis)
    for t in tensors:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError("reconstruct needs CUDA tensors (there is no CPU path)")
        if t.dtype not in _FLOATS:
            raise TypeError(f"reconstruct computes in float32; got {t.dtype}")
        if t.device != source.device:
            raise ValueError("source, metadata, base and basis must be on one device")
    if source.requires_grad:
        raise ValueError("gradients with respect to the source are not computed")
    if tuple(base.shape) != (25, 4) or tuple(basis.shape) != (25, 16, 4):
        raise ValueError("Expected base [25, 4] and basis [25, 16, 4]")
    dtype = torch.promote_types(source.dtype, base.dtype)
    with torch.autocast(device_type="cuda", enabled=False):
        args = [t.to(torch.float32).contiguous() for t in tensors]
        out = _Reconstruct.apply(*args, int(trim), int(gradient_stride), int(phase))
    return out if dtype == torch.float32 else out.to(dtype)


__all__ = ["reconstruct"]

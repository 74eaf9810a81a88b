"""PNG egress and ingress on the GPU.

Egress: the files ``save_rgb`` writes (aeisu/runtime.py:23-27), encoded by the C ABI's
``aeisu_png_encode`` from frames already on the device (or copied there).

``encode_png(frames)`` takes uint8 HWC frames (``[H, W, 3]`` or ``[n, H, W, 3]``, what
``upscale_u8`` returns) or float32 CHW images (``[3, H, W]`` or ``[n, 3, H, W]``, what ``upscale``
returns; quantised as ``save_rgb`` does: clamp to [0, 1], floor(x * 255 + 0.5)) and returns the
PNG file bytes (one ``bytes`` object per frame for a batch).  The decoded pixels are exactly
``save_rgb``'s; the compressed stream is this encoder's own (dynamic Huffman blocks with greedy LZ77 matches), so the
files are byte-for-byte different from PIL's and typically somewhat larger.  ``save_png`` writes
one file.

Ingress: ``decode_png(files)`` is ``read_rgb`` (aeisu/runtime.py:17-20: PIL open,
``convert("RGB")``, uint8 HWC) for one PNG file or a batch of same-sized files, decoded by
``aeisu_png_decode`` (chunks parsed and CRC-checked on the host as PIL checks them; inflate,
unfilter, Adler-32 and RGB conversion on the GPU).  8-bit grey, RGB, palette, grey + alpha and RGBA files, not
interlaced; the pixels equal PIL's.  ``png_info`` reads a file's size and colour type,
``load_png`` reads and decodes one file.  There is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

from . import _lib
from .runtime import CUDA_STREAM_LEGACY, _Array, _device_index

PNG_U8, PNG_F32 = 0, 1


def _kind(frames):
    name = str(getattr(frames, "dtype", "")).replace("torch.", "")
    if name == "uint8":
        return PNG_U8
    if name == "float32":
        return PNG_F32
    raise TypeError(f"encode_png expects uint8 HWC or float32 CHW frames, got {name or type(frames)}")


def encode_png(frames, device="cuda"):
    """PNG file bytes of one frame, or a list of them for a batch (see the module docstring)."""
    kind = _kind(frames)
    nd = frames.ndim
    if kind == PNG_U8:
        if nd not in (3, 4) or frames.shape[-1] != 3:
            raise ValueError(f"Expected uint8 frames [H,W,3] or [n,H,W,3], got {tuple(frames.shape)}")
        h, w = frames.shape[-3], frames.shape[-2]
    else:
        if nd not in (3, 4) or frames.shape[-3] != 3:
            raise ValueError(f"Expected float32 CHW images [3,H,W] or [n,3,H,W], got {tuple(frames.shape)}")
        h, w = frames.shape[-2], frames.shape[-1]
    single = nd == 3
    n = 1 if single else frames.shape[0]
    dev = frames.device.index if getattr(frames, "is_cuda", False) else _device_index(device)
    a = _Array(frames, np.uint8 if kind == PNG_U8 else np.float32, dev)
    lib = _lib.lib()
    bound = int(lib.aeisu_png_bound(h, w))
    if bound == 0:
        raise ValueError("image is empty")
    out = np.empty(n * bound, np.uint8)
    sizes = np.zeros(n, np.uint64)
    _lib.check(lib.aeisu_png_encode(a.ptr, kind, n, h, w, _lib.IO_DEVICE if a.device else _lib.IO_HOST, dev,
                                    out.ctypes.data, out.size, sizes.ctypes.data, a.stream))
    files, at = [], 0
    for s in sizes.tolist():
        files.append(out[at:at + int(s)].tobytes())
        at += int(s)
    return files[0] if single else files


def save_png(path, image, device="cuda"):
    """save_rgb(path, image) with the PNG encoded on the GPU."""
    data = encode_png(image, device)
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_bytes(data)


def png_info(data):
    """(height, width, colour type) of one PNG file's bytes; raises for a broken or unsupported
    file (see ``aeisu_png_info``)."""
    buf = np.frombuffer(bytes(data), np.uint8)
    h, w, color = C.c_int(), C.c_int(), C.c_int()
    _lib.check(_lib.lib().aeisu_png_info(buf.ctypes.data, buf.size, C.byref(h), C.byref(w), C.byref(color)))
    return h.value, w.value, color.value


def decode_png(files, device="cuda", out="host"):
    """uint8 RGB HWC pixels of one PNG file (``bytes``) or ``[n, H, W, 3]`` of a list of
    same-sized files.  ``out="host"`` returns a new numpy array, ``out="device"`` a new torch
    tensor on the GPU; an existing C-contiguous uint8 numpy array or CUDA tensor of the result's
    shape is filled and returned (a caller decoding batch after batch reuses one).  The decode
    runs on the GPU either way."""
    single = isinstance(files, (bytes, bytearray, memoryview))
    batch = [bytes(files)] if single else [bytes(f) for f in files]
    if not batch:
        raise ValueError("no files to decode")
    h, w, _ = png_info(batch[0])
    n = len(batch)
    shape = (h, w, 3) if single else (n, h, w, 3)
    sizes = np.array([len(f) for f in batch], np.uint64)
    offsets = np.zeros(n, np.uint64)
    offsets[1:] = np.cumsum(sizes)[:-1]
    blob = np.frombuffer(b"".join(batch), np.uint8)
    dev = _device_index(device)
    stream = None
    if isinstance(out, str):
        if out == "host":
            result = np.empty(shape, np.uint8)
        elif out == "device":
            import torch
            result = torch.empty(shape, dtype=torch.uint8, device=f"cuda:{dev}")
        else:
            raise ValueError(f"out must be 'host', 'device' or an array, got {out!r}")
    else:
        result = out
    if isinstance(result, np.ndarray):
        if result.dtype != np.uint8 or result.shape != shape or not result.flags.c_contiguous:
            raise ValueError(f"out must be a C-contiguous uint8 array of shape {shape}")
        ptr, flags = result.ctypes.data, _lib.IO_HOST
    else:
        import torch
        if not (isinstance(result, torch.Tensor) and result.is_cuda and result.dtype == torch.uint8
                and tuple(result.shape) == shape and result.is_contiguous()):
            raise ValueError(f"out must be a contiguous uint8 CUDA tensor of shape {shape}")
        dev = result.device.index
        ptr, flags = result.data_ptr(), _lib.IO_DEVICE
        stream = torch.cuda.current_stream(result.device).cuda_stream or CUDA_STREAM_LEGACY
    _lib.check(_lib.lib().aeisu_png_decode(blob.ctypes.data, offsets.ctypes.data, sizes.ctypes.data, n, h, w,
                                           flags, dev, ptr, stream))
    return result


def load_png(path, device="cuda"):
    """read_rgb(path) with the PNG decoded on the GPU (uint8 HWC numpy array)."""
    return decode_png(Path(path).read_bytes(), device)

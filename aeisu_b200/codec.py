"""PNG egress on the GPU: the files ``save_rgb`` writes (aeisu/runtime.py:23-27), encoded by the
C ABI's ``aeisu_png_encode`` from frames already on the device (or copied there).

``encode_png(frames)`` takes uint8 HWC frames (``[H, W, 3]`` or ``[n, H, W, 3]``, what
``upscale_u8`` returns) or float32 CHW images (``[3, H, W]`` or ``[n, 3, H, W]``, what ``upscale``
returns; quantised as ``save_rgb`` does: clamp to [0, 1], floor(x * 255 + 0.5)) and returns the
PNG file bytes (one ``bytes`` object per frame for a batch).  The decoded pixels are exactly
``save_rgb``'s; the compressed stream is this encoder's own (dynamic Huffman blocks with greedy LZ77 matches), so the
files are byte-for-byte different from PIL's and typically somewhat larger.  ``save_png`` writes
one file.  There is no CPU fallback.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

from . import _lib
from .runtime import _Array, _device_index

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

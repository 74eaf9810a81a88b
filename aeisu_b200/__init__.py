"""aeisu_b200: B200-native (sm_100a) AEISU 2x inference behind a C ABI (include/aeisu.h).

The operator surface mirrors the reference's ``aeisu.runtime`` (``load_model``,
``upscale``, ``read_rgb``, ``save_rgb``) and adds batched uint8 ``upscale_u8``.
All arithmetic runs in the in-tree CUDA library ``libaeisu_b200.so``.
"""
from .runtime import Model, load_model, read_rgb, save_rgb, upscale, upscale_u8  # noqa: F401

__all__ = ["Model", "load_model", "read_rgb", "save_rgb", "upscale", "upscale_u8"]

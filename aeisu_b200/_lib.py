"""ctypes binding of the C ABI declared in include/aeisu.h.

The shared library is built in-tree (``python -m aeisu_b200.build``).  There is no CPU
fallback: if the library is missing or cannot load, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libaeisu_b200.so"

OK, INVALID_ARG, BAD_ARTIFACT, CUDA, NONFINITE, TIMEOUT, UNSUPPORTED, OOM = range(8)
PRECISIONS = {"fp32": 0, "fp16": 1, "mixed": 2, "int8": 3}
IO_HOST, IO_DEVICE = 0, 1
FOLDED_VALUES = 115996


class AeisuError(RuntimeError):
    """A failure reported by the library (status code + message)."""

    def __init__(self, status, message):
        super().__init__(f"[aeisu status {status}] {message}")
        self.status = status


class ArtifactError(AeisuError, ValueError):
    pass


class Timings(C.Structure):
    _fields_ = [("analysis_project_ms", C.c_float), ("compress_core_ms", C.c_float),
                ("expand_ms", C.c_float), ("refine_tail_ms", C.c_float),
                ("reconstruction_ms", C.c_float), ("total_ms", C.c_float), ("detailed", C.c_int)]


class Int8Artifact(C.Structure):
    """aeisu_int8_artifact of include/aeisu.h: the shader_precision_v1 arrays."""
    _fields_ = [
        ("analysis", C.c_void_p), ("base", C.c_void_p), ("bank", C.c_void_p),
        ("project_w", C.c_void_p), ("refine_w", C.c_void_p), ("tail_w", C.c_void_p),
        ("project_b", C.c_void_p), ("refine_b", C.c_void_p), ("tail_b", C.c_void_p),
        ("int8_w", C.c_void_p * 6), ("int8_factor", C.c_void_p * 6), ("int8_bias", C.c_void_p * 6),
        ("activation_scales", C.c_void_p),
    ]


_SIGNATURES = {
    "aeisu_open_int8": (C.c_int, [C.POINTER(Int8Artifact), C.c_int, C.POINTER(C.c_void_p)]),
    "aeisu_open_spyr8": (C.c_int, [C.c_char_p, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "aeisu_validate_spyr8": (C.c_int, [C.c_void_p, C.c_size_t, C.c_char_p]),
    "aeisu_open_spyr8_memory": (C.c_int, [C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "aeisu_open_spyr8_headroom": (C.c_int, [C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_float,
                                            C.POINTER(C.c_void_p)]),
    "aeisu_open_folded": (C.c_int, [C.c_void_p, C.c_size_t, C.c_float, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "aeisu_open_sibling": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "aeisu_close": (None, [C.c_void_p]),
    "aeisu_upscale_u8": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                   C.c_uint, C.c_void_p]),
    "aeisu_upscale_f32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                    C.c_uint, C.c_void_p]),
    "aeisu_upscale_u8_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                           C.c_void_p]),
    "aeisu_upscale_u8_band": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                        C.c_uint, C.c_void_p]),
    "aeisu_forward_f32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_uint,
                                    C.c_void_p]),
    "aeisu_predict_coefficients": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                             C.c_uint, C.c_void_p]),
    "aeisu_activation_stats": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_uint, C.c_void_p,
                                         C.c_void_p, C.c_void_p]),
    "aeisu_distortion": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint, C.c_int,
                                   C.c_void_p, C.c_void_p]),
    "aeisu_png_encode": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_uint, C.c_int,
                                   C.c_void_p, C.c_uint64, C.c_void_p, C.c_void_p]),
    "aeisu_png_bound": (C.c_uint64, [C.c_int, C.c_int]),
    "aeisu_png_info": (C.c_int, [C.c_void_p, C.c_uint64, C.POINTER(C.c_int), C.POINTER(C.c_int),
                                 C.POINTER(C.c_int)]),
    "aeisu_png_decode": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_uint,
                                   C.c_int, C.c_void_p, C.c_void_p]),
    "aeisu_reconstruct_f32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                        C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "aeisu_reconstruct_backward_f32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                                 C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                                 C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "aeisu_synchronize": (C.c_int, [C.c_void_p, C.c_void_p, C.c_double]),
    "aeisu_tensor_peak": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_double)]),
    "aeisu_timings_get": (C.c_int, [C.c_void_p, C.POINTER(Timings)]),
    "aeisu_set_detailed_timing": (C.c_int, [C.c_void_p, C.c_int]),
    "aeisu_set_fused_head": (C.c_int, [C.c_void_p, C.c_int]),
    "aeisu_set_timeout": (C.c_int, [C.c_void_p, C.c_double]),
    "aeisu_set_workspace_limit": (C.c_int, [C.c_void_p, C.c_uint64]),
    "aeisu_report": (C.c_char_p, [C.c_void_p]),
    "aeisu_device_bytes": (C.c_uint64, [C.c_void_p]),
    "aeisu_kernel_launches": (C.c_uint64, [C.c_void_p]),
    "aeisu_last_error": (C.c_char_p, []),
    "aeisu_version": (C.c_char_p, []),
}

_lib = None


def lib():
    """Load the library once; raise loudly if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"aeisu_b200 CUDA library not found at {LIB_PATH}; build it with "
                "`python -m aeisu_b200.build` (there is no CPU fallback)")
        handle = C.CDLL(os.fspath(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    return lib().aeisu_last_error().decode()


def check(status: int) -> None:
    if status == OK:
        return
    msg = last_error()
    if status == INVALID_ARG:
        raise ValueError(msg)
    if status == NONFINITE:
        raise FloatingPointError(msg)
    if status == TIMEOUT:
        raise TimeoutError(msg)
    if status == BAD_ARTIFACT:
        raise ArtifactError(status, msg)
    if status == OOM:
        raise MemoryError(msg)
    raise AeisuError(status, msg)

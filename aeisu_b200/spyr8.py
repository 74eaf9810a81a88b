"""SPYR8 v1 artifact container (the reference's ``adaptive_fp8.bin`` layout) in Python.

Layout restated from the reference loader optimized/native/src/neural/srcpyr/SrcPyrModel.cpp
(header struct 37-68, descriptor struct 70-80, validation 243-470) and SrcPyrArchitecture.h
(dtype / layout enums 68-86).  ``read_spyr8`` parses an artifact into numpy arrays,
``write_spyr8`` serialises named tensors with the same header, 64-byte payload alignment
and SHA-256 (computed with the checksum field zeroed).  The runtime's authoritative
parser and validator is the C++ loader behind ``aeisu_open_spyr8``.

Also the OCP FP8 E4M3 ("fn", finite-only) codec used for weights and activations:
round-to-nearest-even with saturation to +-448, as ``__nv_fp8_e4m3(float)`` converts.
"""
from __future__ import annotations

import hashlib
import struct

import numpy as np

MAGIC = b"SPYR8F8\0"
ARCHITECTURE = "aif16x5_learnedrgb4dir8_s32_parallel32x4_learnedbase_oc25_v1"
HEADER_SIZE, DESCRIPTOR_SIZE, ALIGN, CHECKSUM_OFFSET = 512, 80, 64, 184
FP8, FP16, FP32 = 1, 2, 3
VECTOR, OIHW, ADAPTIVE_BASIS = 1, 2, 4
LAYER_NAMES = ("project", "compress", "bottleneck0", "bottleneck1", "bottleneck2", "bottleneck3",
               "expand", "refine", "tail")
LAYER_SHAPES = {"project": (32, 32, 1, 1), "compress": (64, 128, 1, 1), "bottleneck0": (64, 32, 3, 3),
                "bottleneck1": (64, 32, 3, 3), "bottleneck2": (64, 32, 3, 3), "bottleneck3": (64, 32, 3, 3),
                "expand": (128, 64, 1, 1), "refine": (64, 32, 3, 3), "tail": (64, 64, 1, 1)}

# ---- FP8 E4M3 codec ---------------------------------------------------------------

_E4M3_POS = np.array([(m / 8.0) * 2.0 ** -6 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7)
                      for e in range(16) for m in range(8)][:127])  # codes 0x00..0x7e


def e4m3_decode(codes):
    codes = np.asarray(codes, np.uint8)
    mag = np.where((codes & 0x7F) == 0x7F, np.nan, _E4M3_POS[np.minimum(codes & 0x7F, 126)])
    return np.where(codes & 0x80, -mag, mag).astype(np.float32)


def e4m3_encode(x):
    """float -> E4M3 codes: nearest value, ties to even code, saturating at +-448, NaN -> 0x7f."""
    x = np.asarray(x, np.float32)
    a = np.minimum(np.abs(x).astype(np.float64), 448.0)
    hi = np.clip(np.searchsorted(_E4M3_POS, a, side="left"), 0, 126)
    lo = np.maximum(hi - 1, 0)
    dlo, dhi = a - _E4M3_POS[lo], _E4M3_POS[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    code = np.where(np.signbit(x), code | 0x80, code)
    return np.where(np.isnan(x), np.uint8(0x7F), code).astype(np.uint8)


def e4m3_round(x):
    return e4m3_decode(e4m3_encode(x))


# ---- container -----------------------------------------------------------------------

def _dtype_of(arr):
    return {np.dtype(np.uint8): FP8, np.dtype(np.float16): FP16, np.dtype(np.float32): FP32}[arr.dtype]


def write_spyr8(tensors, architecture=ARCHITECTURE, edge_phase_max_shift=0.0, edge_gate_gain=0.0):
    """Serialise ``{name: (array, layout)}`` (uint8 = E4M3 codes, float16, float32)."""
    names = list(tensors)
    count = len(names)
    toc_bytes = count * DESCRIPTOR_SIZE
    payload = (HEADER_SIZE + toc_bytes + ALIGN - 1) // ALIGN * ALIGN
    offsets, cursor = [], payload
    for name in names:
        arr = np.ascontiguousarray(tensors[name][0])
        offsets.append(cursor)
        cursor = (cursor + arr.nbytes + ALIGN - 1) // ALIGN * ALIGN
    size = cursor
    blob = bytearray(size)
    header = struct.pack(
        "<8sIIII64s14I2f4Q", MAGIC, 1, HEADER_SIZE, 0x01020304, 0,
        architecture.encode().ljust(64, b"\0"), 8, 32, 32, 64, 4, 64, 2, 1, 1, OIHW, 1,
        count, ALIGN, DESCRIPTOR_SIZE, edge_phase_max_shift, edge_gate_gain,
        size, HEADER_SIZE, toc_bytes, payload)
    blob[:len(header)] = header
    for i, name in enumerate(names):
        arr, layout = tensors[name]
        arr = np.ascontiguousarray(arr)
        shape = list(arr.shape) + [0] * (4 - arr.ndim)
        desc = struct.pack("<32sIII4IQQ4s", name.encode().ljust(32, b"\0"), _dtype_of(arr), layout,
                           arr.ndim, *shape, offsets[i], arr.nbytes, b"\0" * 4)
        o = HEADER_SIZE + i * DESCRIPTOR_SIZE
        blob[o:o + DESCRIPTOR_SIZE] = desc
        blob[offsets[i]:offsets[i] + arr.nbytes] = arr.tobytes()
    blob[CHECKSUM_OFFSET:CHECKSUM_OFFSET + 32] = hashlib.sha256(bytes(blob)).digest()
    return bytes(blob)


def checksum(data: bytes) -> str:
    z = bytearray(data)
    z[CHECKSUM_OFFSET:CHECKSUM_OFFSET + 32] = b"\0" * 32
    return hashlib.sha256(bytes(z)).hexdigest()


def read_spyr8(data: bytes):
    """Parse an artifact into ``{name: array}`` (E4M3 codes stay uint8).  Light checks only."""
    if data[:8] != MAGIC:
        raise ValueError("not a SPYR8 artifact")
    count, = struct.unpack_from("<I", data, 132)
    out = {}
    for i in range(count):
        o = HEADER_SIZE + i * DESCRIPTOR_SIZE
        name, dtype, layout, rank, s0, s1, s2, s3, off, nbytes, _ = struct.unpack_from(
            "<32sIII4IQQ4s", data, o)
        name = name.split(b"\0", 1)[0].decode()
        shape = (s0, s1, s2, s3)[:rank]
        np_dtype = {FP8: np.uint8, FP16: np.float16, FP32: np.float32}[dtype]
        out[name] = np.frombuffer(data, np_dtype, int(np.prod(shape)), off).reshape(shape).copy()
    return out


def folded_state_from_spyr8(t):
    """Folded-checkpoint view of a SPYR8 artifact: FP16 weights upcast to FP32, FP32 biases,
    the stencil split back into the six analysis tensors; ``basis`` stays projected
    ([25,16,4]) and is returned separately because the artifact does not hold basis_raw."""
    st = t["analysis_stencil"]
    state = {
        "analysis_rgb_basis": st[0:9].reshape(3, 3), "analysis_rgb_mix": st[9:12],
        "analysis_dx_rows": st[12:15], "analysis_dy_cols": st[15:18],
        "analysis_diag45": st[18:21], "analysis_diag135": st[21:24],
        "base_kernel": t["adaptive_base"],
    }
    ref = {"project": "project_540", "compress": "compress_270", "expand": "expand_270",
           "refine": "refine_540", "tail": "metadata_head"}
    for name, key in ref.items():
        state[f"{key}.weight"] = t[f"{name}.weight_fp16"].astype(np.float32)
        state[f"{key}.bias"] = t[f"{name}.bias"]
    for i in range(4):
        w = t[f"bottleneck{i}.weight_fp16"].astype(np.float32)
        b = t[f"bottleneck{i}.bias"]
        state[f"bottleneck_270_a{i + 1}.weight"], state[f"bottleneck_270_b{i + 1}.weight"] = w[:32], w[32:]
        state[f"bottleneck_270_a{i + 1}.bias"], state[f"bottleneck_270_b{i + 1}.bias"] = b[:32], b[32:]
    return state, t["adaptive_basis"]

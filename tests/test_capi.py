"""Host-side checks of the C ABI: the library builds, loads, exports every declared symbol,
and the SPYR8 parser/validator behaves like the reference loader (no GPU needed)."""
import ctypes as C
import hashlib
import re

import numpy as np
import pytest

from conftest import ROOT, staged
from aeisu_b200 import _lib, build, spyr8
from aeisu_b200.synthetic import make_frame, random_folded_state


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.lib()


def declared_functions():
    text = (ROOT / "include" / "aeisu.h").read_text()
    return sorted(set(re.findall(r"^(?:int|void|uint64_t|const char\*)\s+(aeisu_\w+)\s*\(", text, re.M)))


def test_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/aeisu.h but not exported"
    assert set(names) <= set(_lib._SIGNATURES), "python binding misses a declared entry point"


def test_version(lib):
    assert b"sm_100a" in lib.aeisu_version()


def validate(lib, data):
    buf = C.create_string_buffer(bytes(data), len(data))
    out = C.create_string_buffer(65)
    status = lib.aeisu_validate_spyr8(buf, len(data), out)
    return status, out.value.decode()


@pytest.fixture(scope="module")
def artifact():
    from spyr8_helpers import build_artifact
    state = random_folded_state(31)
    return build_artifact(state, [make_frame(5, 32, 40)])


def test_validate_synthetic_artifact(lib, artifact):
    status, digest = validate(lib, artifact)
    assert status == _lib.OK, _lib.last_error()
    assert digest == spyr8.checksum(artifact)


def test_validate_rejects_corruption(lib, artifact):
    bad = bytearray(artifact)
    bad[-70] ^= 0x40  # payload byte: checksum mismatch
    status, _ = validate(lib, bad)
    assert status == _lib.BAD_ARTIFACT and "checksum" in _lib.last_error()
    bad = bytearray(artifact)
    bad[0:8] = b"SPYR9F8\0"
    assert validate(lib, bad)[0] == _lib.BAD_ARTIFACT
    assert validate(lib, artifact[:400])[0] == _lib.BAD_ARTIFACT
    assert validate(lib, artifact[:-64])[0] == _lib.BAD_ARTIFACT


def test_validate_rejects_unknown_architecture(lib):
    from spyr8_helpers import build_artifact
    t = spyr8.read_spyr8(build_artifact(random_folded_state(2), [make_frame(1, 32, 32)]))
    data = spyr8.write_spyr8({k: (v, spyr8.VECTOR if v.ndim == 1 else (spyr8.OIHW if v.ndim == 4 else
                                                                        spyr8.ADAPTIVE_BASIS)) for k, v in t.items()},
                             architecture="aif16x5_feat8_s32_64_v1")
    assert validate(lib, data)[0] == _lib.UNSUPPORTED


def test_validate_rejects_basis_contract(lib):
    from spyr8_helpers import build_artifact
    state = random_folded_state(4)
    basis = np.ones((25, 16, 4), np.float32) * 0.1  # DC != 0
    data = build_artifact(state, [make_frame(1, 32, 32)], {"adaptive_basis": (basis, spyr8.ADAPTIVE_BASIS)})
    status, _ = validate(lib, data)
    assert status == _lib.BAD_ARTIFACT and "zero-DC" in _lib.last_error()


def test_validate_rejects_missing_tensor(lib):
    from spyr8_helpers import build_artifact
    t = spyr8.read_spyr8(build_artifact(random_folded_state(4), [make_frame(1, 32, 32)]))
    del t["tail.bias_fp8"]
    t["extra_pad"] = np.zeros(1, np.float32)  # keep the tensor count at 59
    lay = {k: (v, spyr8.OIHW if v.ndim == 4 else spyr8.ADAPTIVE_BASIS if k.startswith("adaptive") else spyr8.VECTOR)
           for k, v in t.items()}
    status, _ = validate(lib, spyr8.write_spyr8(lay))
    assert status == _lib.BAD_ARTIFACT and "tail.bias_fp8" in _lib.last_error()


def test_reference_artifact_validates(lib):
    path = staged("adaptive_fp8.bin")
    data = path.read_bytes()
    status, digest = validate(lib, data)
    assert status == _lib.OK, _lib.last_error()
    assert digest == data[184:216].hex()
    assert hashlib.sha256(data).hexdigest().startswith("8a6ebf70")


def test_python_writer_reproduces_reference_artifact():
    path = staged("adaptive_fp8.bin")
    data = path.read_bytes()
    t = spyr8.read_spyr8(data)
    layouts = {}
    for i in range(len(t)):
        o = 512 + i * 80
        layouts[data[o:o + 32].split(b"\0")[0].decode()] = int.from_bytes(data[o + 36:o + 40], "little")
    assert spyr8.write_spyr8({k: (v, layouts[k]) for k, v in t.items()}) == data


def test_open_reports_status_without_gpu(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    flat = np.zeros(_lib.FOLDED_VALUES, np.float32)
    h = C.c_void_p()
    status = lib.aeisu_open_folded(flat.ctypes.data, flat.size, 0.5, 0, 0, C.byref(h))
    assert status in (_lib.CUDA, _lib.INVALID_ARG) and not h.value
    assert _lib.last_error()


def test_open_rejects_bad_arguments(lib):
    h = C.c_void_p()
    flat = np.zeros(10, np.float32)
    assert lib.aeisu_open_folded(flat.ctypes.data, 10, 0.5, 0, 0, C.byref(h)) == _lib.INVALID_ARG
    flat = np.zeros(_lib.FOLDED_VALUES, np.float32)
    assert lib.aeisu_open_folded(flat.ctypes.data, flat.size, 0.5, 2, 0, C.byref(h)) == _lib.UNSUPPORTED
    flat[5] = np.inf
    assert lib.aeisu_open_folded(flat.ctypes.data, flat.size, 0.5, 0, 0, C.byref(h)) == _lib.BAD_ARTIFACT
    assert lib.aeisu_upscale_u8(None, None, 1, 8, 8, 0, None, 0, None) == _lib.INVALID_ARG

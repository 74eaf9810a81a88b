"""The INT8/FP16 artifact (shader_precision_v1) on the host: the loader's checks, which follow
MixedRuntime.__init__ (optimized/shader/runtime.py:37-43), the C ABI's array validation, which
runs before any CUDA call, and the int8 restatement in oracle/mixed_np.py (its quantiser and its
distance from the FP32 route, which tests/test_oracle_golden.py pins to the reference)."""
import ctypes as C

import numpy as np
import pytest

from conftest import staged
from oracle import aeisu_np as O
from oracle import mixed_np as M
from aeisu_b200 import _lib
from aeisu_b200.runtime import INT8_LAYERS, int8_arrays
from aeisu_b200.synthetic import make_frame


def record():
    import torch
    return torch.load(staged("aeisu_int8_fp16.pt"), map_location="cpu", weights_only=True)


def test_arrays_and_shapes():
    a = int8_arrays(record())
    assert a["project_w"].dtype == np.uint16 and a["refine_w"].shape == (64, 32, 3, 3)
    assert a["compress.w"].shape == (64, 128, 1, 1) and a["expand.w"].shape == (128, 64, 1, 1)
    for name in INT8_LAYERS:
        assert a[f"{name}.w"].dtype == np.int8 and np.abs(a[f"{name}.w"].astype(int)).max() <= 127
        assert (a[f"{name}.factor"] > 0).all()
    assert (a["activation_scales"] > 0).all()


@pytest.mark.parametrize("change", ["format", "policy", "all_int8"])
def test_rejects_other_policies(change):
    rec = dict(record())
    if change == "format":
        rec["format"] = "shader_precision_v0"
    elif change == "policy":
        rec["precision_policy"] = dict(rec["precision_policy"], refine="int8")
    else:
        rec["all_int8"] = True
    with pytest.raises(ValueError, match="only the published mixed INT8/FP16 policy"):
        int8_arrays(rec)


def _struct(a):
    st = _lib.Int8Artifact()
    for key in ("analysis", "base", "bank", "project_w", "refine_w", "tail_w", "project_b", "refine_b",
                "tail_b", "activation_scales"):
        setattr(st, key, a[key].ctypes.data)
    for i, name in enumerate(INT8_LAYERS):
        st.int8_w[i] = a[f"{name}.w"].ctypes.data
        st.int8_factor[i] = a[f"{name}.factor"].ctypes.data
        st.int8_bias[i] = a[f"{name}.bias"].ctypes.data
    return st


@pytest.mark.parametrize("fault, message", [
    ("code", "outside \\[-127, 127\\]"),
    ("scale", "activation scales must be positive"),
    ("nan", "non-finite"),
    ("missing", "missing"),
])
def test_c_abi_validates_the_arrays_before_any_cuda_call(fault, message):
    a = {k: v.copy() for k, v in int8_arrays(record()).items()}
    if fault == "code":
        a["bottleneck2.w"].reshape(-1)[5] = -128
    elif fault == "scale":
        a["activation_scales"][4] = 0.0
    elif fault == "nan":
        a["expand.factor"][3] = np.nan
    st = _struct(a)
    if fault == "missing":
        st.int8_bias[1] = None
    h = C.c_void_p()
    status = _lib.lib().aeisu_open_int8(C.byref(st), 0, C.byref(h))
    assert status == _lib.BAD_ARTIFACT and not h.value
    assert __import__("re").search(message, _lib.last_error())


def test_int8_code_rounds_half_to_even_and_saturates():
    x = np.array([-200, -127.5, -126.5, -2.5, -0.5, 0.5, 1.5, 2.5, 126.5, 127.5, 3e9], np.float32)
    np.testing.assert_array_equal(M.int8_code(x), [-127, -127, -126, -2, -0., 0, 2, 2, 126, 127, 127])


def test_restatement_is_close_to_the_fp32_route():
    q = M.QuantizedModel(M.int8_record_tensors(record()), "int8")
    ref = O.load_folded(staged("aeisu_area.pt"))
    src = O.u8_to_chw(make_frame(2000, 96, 96))
    p = O.psnr(np.clip(O.upscale(q, src, 0), 0, 1), np.clip(O.upscale(ref, src, 0), 0, 1))
    assert 40.0 <= p < 80.0, p

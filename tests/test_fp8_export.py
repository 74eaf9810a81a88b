"""FP8 exporter (aeisu_b200/fp8_export.py), host side: basis projection, per-channel E4M3
weight quantisation, bias correction and the artifact container, without a GPU."""
import ctypes as C

import numpy as np
import pytest

from conftest import staged
from oracle import aeisu_np as O
from aeisu_b200 import _lib, spyr8
from aeisu_b200 import fp8_export as X
from aeisu_b200.synthetic import random_folded_state


def test_project_basis_matches_the_oracle():
    raw = np.random.default_rng(5).normal(size=(16, 4, 25)).astype(np.float32)
    np.testing.assert_allclose(X.project_basis(raw), O.project_basis(raw), rtol=0, atol=2e-7)
    z = X.project_basis(np.zeros_like(raw))
    assert np.all(z == 0)


def test_weight_quantisation_is_per_channel_e4m3():
    w = np.random.default_rng(6).normal(size=(64, 32, 3, 3)).astype(np.float32)
    w[3] *= 1e-3   # channels of very different magnitude keep their own scale
    codes, scale = X.quantize_weight(w)
    assert codes.dtype == np.uint8 and codes.shape == w.shape and scale.shape == (64,)
    np.testing.assert_allclose(scale, np.abs(w).reshape(64, -1).max(1) / 448, rtol=1e-6)
    deq = spyr8.e4m3_decode(codes) * scale[:, None, None, None]
    # E4M3 keeps 3 mantissa bits: relative error <= 2^-4 for normal values
    big = np.abs(w) > scale[:, None, None, None] * 2 ** -6 * 8
    assert np.all(np.abs(deq - w)[big] <= np.abs(w)[big] * 2 ** -4 * 1.0001)
    # the largest element of every channel maps to +-448
    idx = np.abs(w).reshape(64, -1).argmax(1)
    assert np.all((codes.reshape(64, -1)[np.arange(64), idx] & 0x7F) == 0x7E)


@pytest.mark.parametrize("shape,groups", [((64, 32, 3, 3), 2), ((64, 128, 1, 1), 1), ((128, 64, 1, 1), 1)])
def test_bias_correction_is_the_mean_output_shift(shape, groups):
    rng = np.random.default_rng(7)
    w = rng.normal(size=shape).astype(np.float32)
    codes, scale = X.quantize_weight(w)
    cin = shape[1] * groups
    means = rng.normal(size=cin).astype(np.float32)
    got = X.bias_correction(w, codes, scale, means)
    deq = spyr8.e4m3_decode(codes).astype(np.float64) * scale[:, None, None, None]
    want = np.zeros(shape[0])
    per = shape[0] // groups
    for o in range(shape[0]):
        g = o // per
        for k in range(shape[1]):
            want[o] += (w[o, k].astype(np.float64) - deq[o, k]).sum() * means[g * shape[1] + k]
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-7)


def _artifact(state, means=None):
    scales = np.linspace(0.001, 0.05, 10).astype(np.float32)
    return X.build_artifact(state, scales, means), scales


def test_artifact_layout_matches_the_reference_artifact():
    ref = spyr8.read_spyr8(staged("adaptive_fp8.bin").read_bytes())
    data, scales = _artifact(random_folded_state(3))
    t = spyr8.read_spyr8(data)
    assert list(t) == list(ref), "tensor order differs from adaptive_fp8.bin"
    for name in t:
        assert t[name].dtype == ref[name].dtype and t[name].shape == ref[name].shape, name
    np.testing.assert_array_equal(t["activation_scales"], scales)
    assert data[:8] == spyr8.MAGIC


def test_artifact_passes_the_runtime_validator_and_checksum():
    state = random_folded_state(4)
    means = np.random.default_rng(8).random(448).astype(np.float32)
    data, _ = _artifact(state, means)
    lib = _lib.lib()
    sha = C.create_string_buffer(65)
    assert lib.aeisu_validate_spyr8(data, len(data), sha) == 0, lib.aeisu_last_error()
    assert sha.value.decode() == spyr8.checksum(data)
    t = spyr8.read_spyr8(data)
    # FP16 layers keep their bias; FP8 layers carry the correction
    np.testing.assert_array_equal(t["project.bias_fp8"], t["project.bias"])
    np.testing.assert_array_equal(t["tail.bias_fp8"], t["tail.bias"])
    assert not np.array_equal(t["compress.bias_fp8"], t["compress.bias"])
    lw = X.layer_weights(state)
    w, b = lw["bottleneck2"]
    corr = X.bias_correction(w, t["bottleneck2.weight_fp8"], t["bottleneck2.weight_scale"], means[256:320])
    np.testing.assert_allclose(t["bottleneck2.bias_fp8"], b + corr, rtol=0, atol=1e-7)
    np.testing.assert_array_equal(t["bottleneck2.weight_fp16"], w.astype(np.float16))
    np.testing.assert_array_equal(t["adaptive_base"], state["base_kernel"])


def test_artifact_rejects_bad_scales():
    state = random_folded_state(5)
    for bad in (np.zeros(10), np.full(10, np.nan), np.ones(9)):
        with pytest.raises(ValueError):
            X.build_artifact(state, bad)

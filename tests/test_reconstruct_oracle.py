"""Pin the numpy restatement of reconstruct's forward and gradients to the reference.

tests/golden/reconstruct_grad.npz holds the reference's own outputs and autograd gradients
(tests/golden/make_reconstruct_golden.py).  The sampled-gradient identity restates
tests/test_reference.py:79-99; the argument checks restate aeisu/reconstruction.py:37-52.
"""
import numpy as np
import pytest

from conftest import GOLDEN
from oracle import reconstruct_np as R

FIX = np.load(GOLDEN / "reconstruct_grad.npz")
CASES = sorted({k.split("/")[0] for k in FIX.files})


def case(name):
    g = {k.split("/")[1]: FIX[k] for k in FIX.files if k.startswith(name + "/")}
    b, h, w, trim, stride, phase = (int(v) for v in g["geom"])
    return g, trim, stride, phase


def rel(a, r):
    return float(np.max(np.abs(a - r)) / max(float(np.max(np.abs(r))), 1e-30))


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_autograd(name):
    g, trim, stride, phase = case(name)
    out = R.reconstruct(g["src"], g["meta"], g["base"], g["basis"], trim=trim)
    assert out.shape == g["out"].shape
    assert rel(out, g["out"]) < 1e-6
    gm, gb, gk = R.reconstruct_backward(g["src"], g["meta"], g["base"], g["basis"], g["grad"], trim, stride, phase)
    assert rel(gm, g["g_meta"]) < 1e-6
    if stride == 0:
        assert gb is None and gk is None and g["g_base"].size == 0 and g["g_basis"].size == 0
    else:
        assert rel(gb, g["g_base"]) < 1e-5
        assert rel(gk, g["g_basis"]) < 1e-5


def test_fixture_covers_every_clamp_branch():
    mags = np.concatenate([np.abs(FIX[k]).ravel() for k in FIX.files if k.endswith("/meta")])
    assert (mags <= 2).any() and ((mags > 2) & (mags < 12)).any() and (mags == 12).any() and (mags > 12).any()


def test_sampled_gradients_equal_masked_dense_loss():
    # tests/test_reference.py:79-99: stride-4 sampled base/basis gradients equal those of a
    # dense loss weighted by the stride**2-scaled mask; coefficient gradients stay dense
    rng = np.random.default_rng(17)
    src = rng.random((1, 3, 8, 12), dtype=np.float32)
    meta = (rng.standard_normal((1, 64, 4, 6)) * .2).astype(np.float32)
    base = (rng.standard_normal((25, 4)) * .01).astype(np.float32)
    basis = (rng.standard_normal((25, 16, 4)) * .01).astype(np.float32)
    target = rng.random((1, 3, 16, 24), dtype=np.float32)
    stride, phase = 4, 5
    pred = R.reconstruct(src, meta, base, basis)
    grad = (2 * (pred - target) / pred.size).astype(np.float32)
    dense = R.reconstruct_backward(src, meta, base, basis, grad, 0, 1, phase)
    sampled = R.reconstruct_backward(src, meta, base, basis, grad, 0, stride, phase)
    mask = np.zeros((8, 12), np.float32)
    mask[phase // stride::stride, phase % stride::stride] = stride ** 2
    masked = R.reconstruct_backward(src, meta, base, basis, grad * mask.repeat(2, 0).repeat(2, 1), 0, 1, phase)
    np.testing.assert_allclose(sampled[0], dense[0], atol=1e-7, rtol=1e-6)
    for i in (1, 2):
        np.testing.assert_allclose(sampled[i], masked[i], atol=2e-7, rtol=2e-6)


@pytest.mark.parametrize("src_shape, meta_shape, trim, stride, phase, message", [
    ((3, 8, 8), (1, 64, 4, 4), 0, 1, 0, "Expected NCHW RGB source"),
    ((1, 4, 8, 8), (1, 64, 4, 4), 0, 1, 0, "Expected NCHW RGB source"),
    ((1, 3, 8, 8), (1, 64, 4, 4), 2, 1, 0, "trim must be zero"),
    ((1, 3, 8, 8), (1, 64, 4, 4), 5, 1, 0, "trim must be zero"),
    ((1, 3, 8, 8), (1, 64, 4, 4), -4, 1, 0, "trim must be zero"),
    ((1, 3, 8, 8), (1, 64, 4, 4), 0, -1, 0, "nonnegative"),
    ((1, 3, 8, 8), (1, 64, 4, 4), 0, 1, -1, "nonnegative"),
    ((1, 3, 8, 8), (1, 64, 4, 4), 8, 1, 0, "geometry is invalid"),
    ((1, 3, 8, 8), (1, 64, 4, 5), 0, 1, 0, "geometry is invalid"),
    ((1, 3, 9, 8), (1, 64, 4, 4), 0, 1, 0, "geometry is invalid"),
])
def test_argument_checks(src_shape, meta_shape, trim, stride, phase, message):
    with pytest.raises(ValueError, match=message):
        R.check_geometry(src_shape, meta_shape, trim, stride, phase)

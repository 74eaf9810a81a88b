"""Training reconstruction on the GPU (aeisu_reconstruct_f32 / aeisu_reconstruct_backward_f32
through aeisu_b200.reconstruction.reconstruct) against the reference's own outputs and autograd
gradients (tests/golden/reconstruct_grad.npz) and the FP32 oracle (oracle/reconstruct_np.py).

Tolerances, relative to the largest magnitude of the expected tensor: 2e-6 for the output and
the metadata gradients, 2e-5 for the base/basis gradients (sums over every sampled pixel, whose
order differs from torch's reductions).  At the training recipe's full size (32 x 288 x 288,
trim 32, stride 16) the checks are size-independent: the reference's sampled-gradient identity
(tests/test_reference.py:79-99), exact scaling of every gradient by a power of two, bit-identical
repeated calls, and coefficient gradients that do not depend on the stride.
"""
import numpy as np
import pytest
import torch

from oracle import reconstruct_np as R
from aeisu_b200.reconstruction import reconstruct
from test_reconstruct_oracle import CASES, case, rel

pytestmark = pytest.mark.gpu


def cuda(a, grad=False):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.requires_grad_() if grad else t


def run(src, meta, base, basis, grad, trim, stride, phase):
    m, b, k = cuda(meta, True), cuda(base, True), cuda(basis, True)
    out = reconstruct(cuda(src), m, b, k, trim=trim, gradient_stride=stride, phase=phase)
    out.backward(cuda(grad))
    torch.cuda.synchronize()
    pull = lambda t: None if t.grad is None else t.grad.cpu().numpy()
    return out.detach().cpu().numpy(), pull(m), pull(b), pull(k)


@pytest.mark.parametrize("name", CASES)
def test_matches_reference_autograd(name):
    g, trim, stride, phase = case(name)
    out, gm, gb, gk = run(g["src"], g["meta"], g["base"], g["basis"], g["grad"], trim, stride, phase)
    assert out.shape == g["out"].shape and rel(out, g["out"]) < 2e-6
    assert rel(gm, g["g_meta"]) < 2e-6
    if stride == 0:
        assert gb is None and gk is None
    else:
        assert rel(gb, g["g_base"]) < 2e-5 and rel(gk, g["g_basis"]) < 2e-5


def inputs(seed, b, h, w, trim):
    rng = np.random.default_rng(seed)
    src = rng.random((b, 3, h, w), dtype=np.float32)
    meta = (rng.standard_normal((b, 64, h // 2, w // 2)) * 2.0).astype(np.float32)
    meta[rng.random(meta.shape) < 0.05] *= 8
    base = (rng.standard_normal((25, 4)) * 0.05).astype(np.float32)
    basis = (rng.standard_normal((25, 16, 4)) * 0.05).astype(np.float32)
    off = trim // 2
    grad = rng.standard_normal((b, 3, 2 * (h - 2 * off), 2 * (w - 2 * off))).astype(np.float32)
    return src, meta, base, basis, grad


@pytest.mark.parametrize("b,h,w,trim,stride,phase", [
    (2, 70, 100, 0, 1, 0),        # several tiles in x, a partial tile in y
    (1, 66, 130, 4, 2, 1),        # core 62 x 126: ragged tiles both ways
    (2, 96, 136, 32, 16, 0),      # the training recipe's trim and stride
    (1, 40, 300, 6, 3, 8),        # odd LR border, wide
    (3, 12, 8, 0, 5, 24),         # a core smaller than one tile
    (1, 2, 2, 0, 1, 0),           # the smallest frame: one metadata pixel
    (1, 10, 6, 4, 1, 0),          # a 6 x 2 core
])
def test_matches_oracle(b, h, w, trim, stride, phase):
    src, meta, base, basis, grad = inputs(b * 7919 + h * 31 + w, b, h, w, trim)
    out, gm, gb, gk = run(src, meta, base, basis, grad, trim, stride, phase)
    assert rel(out, R.reconstruct(src, meta, base, basis, trim)) < 2e-6
    wm, wb, wk = R.reconstruct_backward(src, meta, base, basis, grad, trim, stride, phase)
    assert rel(gm, wm) < 2e-6
    assert rel(gb, wb) < 2e-5 and rel(gk, wk) < 2e-5


def test_border_metadata_gradients_are_zero():
    src, meta, base, basis, grad = inputs(3, 1, 40, 48, 8)
    _, gm, _, _ = run(src, meta, base, basis, grad, 8, 1, 0)
    full = np.abs(R.unpack_coefficients(gm))   # gradient per LR pixel (clamp keeps zeros zero)
    core = np.zeros(full.shape[2:], bool)
    core[4:36, 4:44] = True
    assert (full[..., ~core] == 0).all() and (full[..., core] != 0).any()


def training_batch(seed=5):
    # the training recipe: batch 32, 512x512 HR targets, source_pad 16 -> 288x288 sources, trim 32
    g = torch.Generator(device="cuda").manual_seed(seed)
    src = torch.rand((32, 3, 288, 288), device="cuda", generator=g)
    meta = torch.randn((32, 64, 144, 144), device="cuda", generator=g) * 2
    base = torch.randn((25, 4), device="cuda", generator=g) * 0.05
    basis = torch.randn((25, 16, 4), device="cuda", generator=g) * 0.05
    grad = torch.randn((32, 3, 512, 512), device="cuda", generator=g)
    return src, meta, base, basis, grad


def grads(src, meta, base, basis, grad, stride, phase, trim=32):
    m, b, k = (t.clone().requires_grad_() for t in (meta, base, basis))
    out = reconstruct(src, m, b, k, trim=trim, gradient_stride=stride, phase=phase)
    out.backward(grad)
    return out.detach(), m.grad, b.grad, k.grad


def test_full_size_sampled_gradient_identity():
    src, meta, base, basis, grad = training_batch()
    stride, phase = 16, 37
    out, gm, gb, gk = grads(src, meta, base, basis, grad, stride, phase)
    assert out.shape == (32, 3, 512, 512) and torch.isfinite(out).all()
    # dense coefficient gradients do not depend on the stride (bit for bit)
    _, gm1, gb1, gk1 = grads(src, meta, base, basis, grad, 1, 0)
    assert torch.equal(gm, gm1)
    # sampled base/basis gradients == dense ones of the stride**2-weighted mask
    ph = phase % stride ** 2
    mask = torch.zeros((256, 256), device="cuda")
    mask[ph // stride::stride, ph % stride::stride] = stride ** 2
    hr = mask.repeat_interleave(2, 0).repeat_interleave(2, 1)
    _, _, gbm, gkm = grads(src, meta, base, basis, grad * hr, 1, 0)
    for a, b_ in ((gb, gbm), (gk, gkm)):
        assert float((a - b_).abs().max()) <= 2e-5 * float(b_.abs().max())


def test_full_size_scaling_and_determinism():
    src, meta, base, basis, grad = training_batch(9)
    first = grads(src, meta, base, basis, grad, 16, 0)
    again = grads(src, meta, base, basis, grad, 16, 0)
    doubled = grads(src, meta, base, basis, grad * 2, 16, 0)
    for a, b_, d in zip(first[1:], again[1:], doubled[1:]):
        assert torch.equal(a, b_)          # deterministic reductions
        assert torch.equal(d, a * 2)       # linear in the upstream gradient, exactly for 2x


def test_stride_zero_leaves_filters_without_gradient():
    src, meta, base, basis, grad = inputs(4, 1, 16, 16, 0)
    out, gm, gb, gk = run(src, meta, base, basis, grad, 0, 0, 0)
    assert gb is None and gk is None and np.abs(gm).max() > 0


def test_bf16_metadata_gradient_dtype():
    src, meta, base, basis, grad = inputs(6, 1, 20, 24, 4)
    m = cuda(meta).to(torch.bfloat16).requires_grad_()
    out = reconstruct(cuda(src), m, cuda(base), cuda(basis), trim=4)
    out.backward(cuda(grad))
    assert out.dtype == torch.float32 and m.grad.dtype == torch.bfloat16
    want, _, _ = R.reconstruct_backward(src, m.detach().float().cpu().numpy(), base, basis, grad, 4, 1, 0)
    got = m.grad.float().cpu().numpy()
    assert rel(got, want) < 1e-2   # bf16 rounding of the gradient itself


@pytest.mark.parametrize("kw, message", [
    (dict(trim=2), "trim must be zero"),
    (dict(trim=3), "trim must be zero"),
    (dict(gradient_stride=-1), "nonnegative"),
    (dict(phase=-2), "nonnegative"),
    (dict(trim=16), "geometry is invalid"),
])
def test_errors_follow_the_reference(kw, message):
    src, meta, base, basis, _ = inputs(8, 1, 16, 16, 0)
    with pytest.raises(ValueError, match=message):
        reconstruct(cuda(src), cuda(meta), cuda(base), cuda(basis), **kw)


def test_refuses_cpu_and_float64():
    src, meta, base, basis, _ = inputs(8, 1, 8, 8, 0)
    with pytest.raises(ValueError, match="CUDA"):
        reconstruct(torch.from_numpy(src), torch.from_numpy(meta), torch.from_numpy(base), torch.from_numpy(basis))
    with pytest.raises(TypeError):
        reconstruct(cuda(src).double(), cuda(meta), cuda(base), cuda(basis))

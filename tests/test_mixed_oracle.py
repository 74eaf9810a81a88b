"""CPU checks of the reduced-precision restatement (oracle/mixed_np.py)."""
import numpy as np
import torch

from conftest import staged
from oracle import aeisu_np as O
from oracle import mixed_np as M
from aeisu_b200 import spyr8
from aeisu_b200.synthetic import make_frame


def test_e4m3_rounding_three_ways():
    x = np.random.default_rng(0).normal(0, 60, 100000).astype(np.float32)
    x = np.concatenate([x, np.float32([0, -0., 448, 450, 464, 465, 1e6, -1e6, 2 ** -9, 2 ** -10,
                                       3 * 2 ** -11, 0.00146484375, 240, 248, 232])])
    ours = M.e4m3(x)
    np.testing.assert_array_equal(ours, spyr8.e4m3_round(x))
    inrange = np.abs(x) <= 448
    ref = torch.from_numpy(x[inrange]).to(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(ours[inrange], ref)
    assert ours[~inrange].tolist() == [448.0 if v > 0 else -448.0 for v in x[~inrange]]
    codes = np.arange(256, dtype=np.uint8)
    a, b = M.e4m3_decode(codes), spyr8.e4m3_decode(codes)
    np.testing.assert_array_equal(np.isnan(a), np.isnan(b))
    np.testing.assert_array_equal(a[~np.isnan(a)], b[~np.isnan(b)])


def test_artifact_fp16_weights_are_the_area_checkpoint():
    # the shipped mixed artifact was exported from aeisu_area.pt (FP16 weights, base, stencil)
    t = spyr8.read_spyr8(staged("adaptive_fp8.bin").read_bytes())
    area = O.load_folded(staged("aeisu_area.pt"))
    state, basis = spyr8.folded_state_from_spyr8(t)
    for k, v in state.items():
        ref = area.state[k]
        tol = 1e-3 * max(1.0, float(np.abs(ref).max())) if k.endswith(".weight") else 1e-6
        np.testing.assert_allclose(v, ref, atol=tol, rtol=0, err_msg=k)
    np.testing.assert_allclose(basis, area.basis, atol=1e-7)


def test_fp16_restatement_is_close_to_fp32():
    t = spyr8.read_spyr8(staged("adaptive_fp8.bin").read_bytes())
    ref = O.load_folded(staged("aeisu_area.pt"))
    src = O.u8_to_chw(make_frame(801, 96, 96))
    assert O.psnr(O.upscale(M.QuantizedModel(t, "fp16"), src, 0), O.upscale(ref, src, 0)) >= 60


def test_own_weights_state_is_the_mixed_routes_weights():
    # FP32 on the mixed route's own weights: the FP8 layers dequantised (E4M3 code x channel scale,
    # bias_fp8).  With the activations left unquantised the mixed restatement's FP8 layers reduce
    # to it, so a frame through the restatement at 2x headroom stays close (activation rounding
    # only), and nearer to it than to FP32 on the FP16 weights
    t = spyr8.read_spyr8(staged("adaptive_fp8.bin").read_bytes())
    state16, basis = spyr8.folded_state_from_spyr8(t)
    own = O.FoldedModel(M.own_weights_state(t, state16), basis=basis)
    w = M.e4m3_decode(t["compress.weight_fp8"]) * t["compress.weight_scale"].reshape(-1, 1, 1, 1)
    np.testing.assert_array_equal(own.state["compress_270.weight"], w.astype(np.float32))
    np.testing.assert_array_equal(own.state["bottleneck_270_b3.bias"], t["bottleneck2.bias_fp8"][32:])
    src = O.u8_to_chw(make_frame(2005, 64, 64))
    mixed = O.upscale(M.QuantizedModel(t, "mixed", headroom=2.0), src, 0)
    p_own = O.psnr(np.clip(mixed, 0, 1), np.clip(O.upscale(own, src, 0), 0, 1))
    p_f16 = O.psnr(np.clip(mixed, 0, 1), np.clip(O.upscale(O.FoldedModel(state16, basis=basis), src, 0), 0, 1))
    assert p_own >= 50 and p_own > p_f16, (p_own, p_f16)

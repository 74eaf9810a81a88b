"""Build SPYR8 artifacts from folded weights for tests (calibrated with the CPU oracle)."""
import numpy as np

from aeisu_b200 import spyr8
from oracle import aeisu_np as O

_SP = {"project": "project_540", "compress": "compress_270", "expand": "expand_270",
       "refine": "refine_540", "tail": "metadata_head"}


def layer_weights(state):
    out = {}
    for name, key in _SP.items():
        out[name] = (state[f"{key}.weight"], state[f"{key}.bias"])
    for i in range(4):
        out[f"bottleneck{i}"] = (
            np.concatenate([state[f"bottleneck_270_a{i + 1}.weight"], state[f"bottleneck_270_b{i + 1}.weight"]]),
            np.concatenate([state[f"bottleneck_270_a{i + 1}.bias"], state[f"bottleneck_270_b{i + 1}.bias"]]))
    return out


def activation_stats(state, frames):
    """CPU restatement of aeisu_activation_stats: per-layer max |x| of the FP32 activations the
    mixed route quantises (activation_scales order) and the FP8 layers' input-channel means
    (compress in unshuffle order c*4 + phase, bottleneck 0-3 and expand), over the padded
    frames, pixels weighted equally."""
    st = O.FoldedModel(state).state
    peaks = np.zeros(10)
    sums = np.zeros(448)
    count = np.zeros(448)
    for frame in frames:
        src = O.u8_to_chw(frame)
        h, w = src.shape[1:]
        py, px, ph, pw = O.pad_geometry(h, w)
        x = np.pad(src[None], ((0, 0), (0, 0), (py, ph - h - py), (px, pw - w - px)), mode="edge")

        def conv(name, v, g=1):
            return O.conv2d(v, st[f"{name}.weight"], st[f"{name}.bias"], g)
        feat = O.feature8(x, st)
        enc = O.leaky(conv("project_540", O.pixel_unshuffle(feat)))
        low = O.leaky(conv("compress_270", O.pixel_unshuffle(enc)))
        vals = [O.pixel_unshuffle(feat), enc, low]
        ins = [O.pixel_unshuffle(enc), low]
        a, b = low[:, :32], low[:, 32:]
        for i in range(1, 5):
            a = O.leaky(conv(f"bottleneck_270_a{i}", a))
            b = O.leaky(conv(f"bottleneck_270_b{i}", b))
            vals.append(np.concatenate([a, b], 1))
            ins.append(vals[-1])
        exp = O.leaky(conv("expand_270", np.concatenate([a, b], 1)))
        dec_in = enc + O.pixel_shuffle(exp)
        dec = O.leaky(conv("refine_540", dec_in))
        vals += [exp, dec_in, dec]
        for k, v in enumerate(vals):
            peaks[k] = max(peaks[k], float(np.abs(v).max()))
        o = 0
        for v in ins:   # compress input, bottleneck 0-3 inputs, expand input
            c = v.shape[1]
            sums[o:o + c] += v.sum(axis=(0, 2, 3), dtype=np.float64)
            count[o:o + c] += v.shape[0] * v.shape[2] * v.shape[3]
            o += c
    return peaks.astype(np.float32), (sums / count).astype(np.float32)


def activation_scales(state, frames):
    """Per-layer absmax/448 of the FP32 activations the mixed route quantises."""
    return (np.maximum(activation_stats(state, frames)[0], 1e-6) / 448.0).astype(np.float32)


def build_artifact(state, frames, tensors_override=None):
    """Serialise a SPYR8 v1 artifact (same tensor order as the reference's adaptive_fp8.bin)."""
    t = {"activation_scales": (activation_scales(state, frames), spyr8.VECTOR)}
    lw = layer_weights(state)
    for name in spyr8.LAYER_NAMES:
        w, b = lw[name]
        w = w.astype(np.float32)
        scale = (np.maximum(np.abs(w).reshape(w.shape[0], -1).max(1), 1e-12) / 448.0).astype(np.float32)
        t[f"{name}.weight_fp8"] = (spyr8.e4m3_encode(w / scale[:, None, None, None]), spyr8.OIHW)
        t[f"{name}.weight_fp16"] = (w.astype(np.float16), spyr8.OIHW)
        t[f"{name}.weight_scale"] = (scale, spyr8.VECTOR)
        t[f"{name}.bias"] = (b.astype(np.float32), spyr8.VECTOR)
        t[f"{name}.prelu"] = (np.full(w.shape[0], 1.0 if name == "tail" else 0.1, np.float32), spyr8.VECTOR)
    for name in spyr8.LAYER_NAMES:
        t[f"{name}.bias_fp8"] = (lw[name][1].astype(np.float32), spyr8.VECTOR)
    t["adaptive_basis"] = (O.project_basis(state["basis_raw"]), spyr8.ADAPTIVE_BASIS)
    t["precision_guards"] = (np.zeros(2, np.float32), spyr8.VECTOR)
    t["adaptive_base"] = (state["base_kernel"].astype(np.float32), spyr8.ADAPTIVE_BASIS)
    stencil = np.concatenate([state["analysis_rgb_basis"].reshape(-1), state["analysis_rgb_mix"],
                              state["analysis_dx_rows"], state["analysis_dy_cols"],
                              state["analysis_diag45"], state["analysis_diag135"]]).astype(np.float32)
    t["analysis_stencil"] = (stencil, spyr8.VECTOR)
    if tensors_override:
        t.update(tensors_override)
    return spyr8.write_spyr8(t)

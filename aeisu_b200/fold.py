"""Fold a training checkpoint into the deployed parameters, as ``load_model`` does for one.

The reference's ``runtime.load_model`` (aeisu/runtime.py:45-56) accepts the checkpoints
train.py writes: when the state holds ``.rep_low_u`` keys it builds the training model
``AEISU`` (aeisu/model.py:37), loads the state strictly and folds it with ``fold_model``
(aeisu/model.py:599-602), i.e. ``AEISU.folded_production_state_dict`` (aeisu/model.py:510-544).
Every training-only coordinate is static with respect to the image, so folding is pure
parameter algebra; this module restates it in numpy (float64 sums, rounded once to float32)
and returns the 34 tensors of ``FoldedAEISU.state_dict()``, which the C ABI then uploads.

Restated pieces, each from its reference definition:

* ``ReparamConv2d.effective_weight`` = weight + ``reparam_addition``
  (aeisu/reparameterization.py:148-175): two low-rank centre paths, the identity path of
  square convolutions, and for 3x3 kernels the centre, row, column, spatial low-rank,
  directional-template and depthwise paths.
* the analysis constants (aeisu/model.py:205-222): learned RGB basis + diagonal + low rank,
  RGB mix + BT.709 and uniform gains, each stencil + seed and curve gains.
* ``_combined_base_kernel`` (aeisu/model.py:224-244) and ``_combined_basis_raw``
  (aeisu/model.py:246-271): the structured 5x5 branches and the 64-way mixed bank.
* the templates of aeisu/reparameterization.py:17-76.
"""
from __future__ import annotations

import numpy as np

F64 = np.float64
LOW_RANK, SECOND_LOW_RANK, SPATIAL_LOW_RANK = 8, 16, 8      # reparameterization.py:10-12
BASIS_MIXED_BANK, BASIS_SEPARABLE_RANK, BASE_EXTRA_BRANCHES = 64, 2, 4   # reparameterization.py:13-15
BT709 = (0.2126, 0.7152, 0.0722)                               # model.py:18
# deployed convolutions (aeisu/model.py:20-28): name, in, out, kernel
CONVOLUTIONS = (
    ("project_540", 32, 32, 1),
    ("compress_270", 128, 64, 1),
    *((f"bottleneck_270_{b}{i}", 32, 32, 3) for b in ("a", "b") for i in range(1, 5)),
    ("expand_270", 64, 128, 1),
    ("refine_540", 32, 64, 3),
    ("metadata_head", 64, 64, 1),
)
# analysis stencils: name, seed values (aeisu/model.py:511-541)
STENCILS = (("dx_rows", "dx", (0.125, 0.25, 0.125)), ("dy_cols", "dy", (0.125, 0.25, 0.125)),
            ("diag45", "diag45", (0.25, 0.125, 0.125)), ("diag135", "diag135", (0.25, 0.125, 0.125)))
CURVE = (0.5, -1.0, 0.5)


def directional_templates():
    """The six L1-normalised 3x3 templates of reparameterization.py:17-27 (dx, dy, d45, d135,
    lap4, lap8), each divided by max(1, sum |t|)."""
    t = np.array([
        [[-1, 0, 1], [-2, 0, 2], [-1, 0, 1]],
        [[-1, -2, -1], [0, 0, 0], [1, 2, 1]],
        [[-2, -1, 0], [-1, 0, 1], [0, 1, 2]],
        [[0, 1, 2], [-1, 0, 1], [-2, -1, 0]],
        [[0, 1, 0], [1, -4, 1], [0, 1, 0]],
        [[1, 1, 1], [1, -8, 1], [1, 1, 1]],
    ], np.float32)
    return t / np.maximum(np.abs(t).sum(axis=(1, 2), keepdims=True), np.float32(1))


def _ring():
    return [(y, x) for y in range(5) for x in range(5) if y in (0, 4) or x in (0, 4)]


def structural_5x5_templates():
    """The eight 5x5 structural templates of reparameterization.py:30-64, L1-normalised."""
    t = np.zeros((8, 5, 5), np.float32)
    t[0, 2, 1], t[0, 2, 3] = -1, 1
    t[1, 1, 2], t[1, 3, 2] = -1, 1
    t[2, 1, 1], t[2, 3, 3] = -1, 1
    t[3, 1, 3], t[3, 3, 1] = 1, -1
    t[4, 2, 2] = -4
    t[4, 1, 2] = t[4, 3, 2] = t[4, 2, 1] = t[4, 2, 3] = 1
    t[5, 1:4, 1:4] = 1
    t[5, 2, 2] = -8
    t[6, 1:4, 1:4] = -1.0 / 8.0
    t[6, 2, 2] = 1
    for y, x in _ring():
        t[7, y, x] = -1.0 / 16.0
    t[7, 2, 2] = 1
    return t / np.maximum(np.abs(t).sum(axis=(1, 2), keepdims=True), np.float32(1))


def outer_ring_templates():
    """One-hot 5x5 templates of the sixteen perimeter taps, row-major (reparameterization.py:67-76)."""
    out = np.zeros((16, 5, 5), np.float32)
    for i, (y, x) in enumerate(_ring()):
        out[i, y, x] = 1
    return out


def _pad(x, left, right, top, bottom):
    """F.pad over the last two dimensions (zeros)."""
    widths = [(0, 0)] * (x.ndim - 2) + [(top, bottom), (left, right)]
    return np.pad(x, widths)


def _diag_embed(v):
    """torch.diag_embed over the last dimension."""
    n = v.shape[-1]
    out = np.zeros(v.shape + (n,), v.dtype)
    idx = np.arange(n)
    out[..., idx, idx] = v
    return out


def conv_keys(cin, cout, k):
    """Parameter names of one ReparamConv2d (reparameterization.py:87-141), in declaration order."""
    keys = ["weight", "bias", "rep_low_u", "rep_low_v", "rep_low2_u", "rep_low2_v"]
    if cin == cout:
        keys.append("rep_identity")
    if k == 3:
        keys += ["rep_center", "rep_row", "rep_col", "rep_spatial_u", "rep_spatial_v", "rep_directional_mix"]
        if cin == cout:
            keys.append("rep_depthwise")
    return keys


def training_shapes():
    """Name -> shape of every tensor in an AEISU training state dict (aeisu/model.py:40-168 and
    reparameterization.py:87-141), in state_dict order."""
    m, r = BASIS_MIXED_BANK, BASIS_SEPARABLE_RANK
    shapes = {}
    shapes.update({
        "analysis_rgb_basis": (3, 3), "analysis_rgb_mix": (3,), "analysis_dx_rows": (3,),
        "analysis_dy_cols": (3,), "analysis_diag45": (3,), "analysis_diag135": (3,),
        "analysis_rgb_basis_diag": (3,), "analysis_rgb_basis_u": (3, 2), "analysis_rgb_basis_v": (2, 3),
        "analysis_rgb_mix_bt709_gain": (), "analysis_rgb_mix_uniform_gain": (),
    })
    for _, short, _ in STENCILS:
        shapes[f"analysis_{short}_seed_gain"] = ()
        shapes[f"analysis_{short}_curve_gain"] = ()
    shapes.update({
        "base_kernel": (25, 4), "base_rep_kernels": (BASE_EXTRA_BRANCHES, 25, 4),
        "base_rep_slopes": (BASE_EXTRA_BRANCHES,), "base_rep_3x3": (4, 3, 3), "base_rep_1x5": (4, 1, 5),
        "base_rep_5x1": (4, 5, 1), "base_rep_1x3": (4, 1, 3), "base_rep_3x1": (4, 3, 1), "base_rep_1x1": (4, 1, 1),
        "base_rep_diag": (4, 5), "base_rep_anti_diag": (4, 5), "base_rep_outer": (4, 16),
        "base_rep_sep_y": (4, r, 5), "base_rep_sep_x": (4, r, 5), "base_rep_template_gain": (4, 8),
        "basis_raw": (16, 4, 25),
        "basis_mix_main": (m, 4, 5, 5), "basis_mix_full": (m, 4, 5, 5), "basis_mix_3x3": (m, 4, 3, 3),
        "basis_mix_1x5": (m, 4, 1, 5), "basis_mix_5x1": (m, 4, 5, 1), "basis_mix_1x3": (m, 4, 1, 3),
        "basis_mix_3x1": (m, 4, 3, 1), "basis_mix_1x1": (m, 4, 1, 1), "basis_mix_diag": (m, 4, 5),
        "basis_mix_anti_diag": (m, 4, 5), "basis_mix_outer": (m, 4, 16), "basis_mix_sep_y": (m, 4, r, 5),
        "basis_mix_sep_x": (m, 4, r, 5), "basis_mix_template_gain": (m, 4, 8), "basis_mix_matrix": (m, 16),
    })
    # the convolution submodules follow the model's own parameters in state_dict order
    for name, cin, cout, k in CONVOLUTIONS:
        r1 = max(1, min(LOW_RANK, cin, cout))
        r2 = max(1, min(SECOND_LOW_RANK, cin, cout))
        rs = max(1, min(SPATIAL_LOW_RANK, cin, cout))
        full = {"weight": (cout, cin, k, k), "bias": (cout,), "rep_low_u": (cout, r1), "rep_low_v": (r1, cin),
                "rep_low2_u": (cout, r2), "rep_low2_v": (r2, cin), "rep_identity": (cout,),
                "rep_center": (cout, cin, 1, 1), "rep_row": (cout, cin, 1, 3), "rep_col": (cout, cin, 3, 1),
                "rep_spatial_u": (cout, rs), "rep_spatial_v": (rs, cin, 3, 3),
                "rep_directional_mix": (6, cout, cin), "rep_depthwise": (cout, 3, 3)}
        for key in conv_keys(cin, cout, k):
            shapes[f"{name}.{key}"] = full[key]
    return shapes


def is_training_state(state) -> bool:
    """runtime.load_model's test for a training checkpoint (aeisu/runtime.py:49)."""
    return any(".rep_low_u" in key for key in state)


def _arrays(state):
    """The state as float64 numpy arrays, checked strictly against the training layout (as
    load_state_dict(strict=True) does, aeisu/runtime.py:51)."""
    shapes = training_shapes()
    missing = [k for k in shapes if k not in state]
    extra = [k for k in state if k not in shapes]
    if missing or extra:
        raise ValueError(f"training checkpoint does not match the AEISU layout: missing {missing[:4]}, "
                         f"unexpected {extra[:4]}")
    out = {}
    for key, shape in shapes.items():
        v = state[key]
        v = v.detach().cpu().numpy() if hasattr(v, "detach") else np.asarray(v)
        if tuple(v.shape) != shape:
            raise ValueError(f"{key}: expected shape {shape}, got {tuple(v.shape)}")
        out[key] = v.astype(F64)
    return out


def _conv_addition(s, name, cin, cout, k):
    """ReparamConv2d.reparam_addition (reparameterization.py:148-172)."""
    p = lambda key: s[f"{name}.{key}"]
    centre = lambda c: c if k == 1 else _pad(c, 1, 1, 1, 1)
    add = centre((p("rep_low_u") @ p("rep_low_v")).reshape(cout, cin, 1, 1))
    add = add + centre((p("rep_low2_u") @ p("rep_low2_v")).reshape(cout, cin, 1, 1))
    eye = np.eye(cout, cin).reshape(cout, cin, 1, 1)
    if cin == cout:
        add = add + centre(eye * p("rep_identity").reshape(-1, 1, 1, 1))
    if k == 3:
        add = add + centre(p("rep_center"))
        add = add + _pad(p("rep_row"), 0, 0, 1, 1)
        add = add + _pad(p("rep_col"), 1, 1, 0, 0)
        add = add + np.einsum("or,rihw->oihw", p("rep_spatial_u"), p("rep_spatial_v"))
        add = add + np.einsum("toi,thw->oihw", p("rep_directional_mix"), directional_templates().astype(F64))
        if cin == cout:
            add = add + eye * p("rep_depthwise")[:, None, :, :]
    return add


def _structured_base(s):
    """AEISU._structured_base_addition_5x5 (aeisu/model.py:224-239): [phase, 5, 5]."""
    out = _pad(s["base_rep_3x3"], 1, 1, 1, 1)
    out = out + _pad(s["base_rep_1x5"], 0, 0, 2, 2)
    out = out + _pad(s["base_rep_5x1"], 2, 2, 0, 0)
    out = out + _pad(s["base_rep_1x3"], 1, 1, 2, 2)
    out = out + _pad(s["base_rep_3x1"], 2, 2, 1, 1)
    out = out + _pad(s["base_rep_1x1"], 2, 2, 2, 2)
    out = out + _diag_embed(s["base_rep_diag"])
    out = out + _diag_embed(s["base_rep_anti_diag"])[..., ::-1]
    out = out + np.einsum("pt,thw->phw", s["base_rep_outer"], outer_ring_templates().astype(F64))
    out = out + np.einsum("pry,prx->pyx", s["base_rep_sep_y"], s["base_rep_sep_x"])
    out = out + np.einsum("pt,thw->phw", s["base_rep_template_gain"], structural_5x5_templates().astype(F64))
    return out


def _basis_bank(s):
    """AEISU._basis_training_bank_5x5 (aeisu/model.py:246-263): [64, 4, 5, 5]."""
    out = s["basis_mix_main"] + s["basis_mix_full"]
    out = out + _pad(s["basis_mix_3x3"], 1, 1, 1, 1)
    out = out + _pad(s["basis_mix_1x5"], 0, 0, 2, 2)
    out = out + _pad(s["basis_mix_5x1"], 2, 2, 0, 0)
    out = out + _pad(s["basis_mix_1x3"], 1, 1, 2, 2)
    out = out + _pad(s["basis_mix_3x1"], 2, 2, 1, 1)
    out = out + _pad(s["basis_mix_1x1"], 2, 2, 2, 2)
    out = out + _diag_embed(s["basis_mix_diag"])
    out = out + _diag_embed(s["basis_mix_anti_diag"])[..., ::-1]
    out = out + np.einsum("mpt,thw->mphw", s["basis_mix_outer"], outer_ring_templates().astype(F64))
    out = out + np.einsum("mpry,mprx->mpyx", s["basis_mix_sep_y"], s["basis_mix_sep_x"])
    out = out + np.einsum("mpt,thw->mphw", s["basis_mix_template_gain"], structural_5x5_templates().astype(F64))
    return out


def fold_training_state(state) -> dict:
    """AEISU.folded_production_state_dict (aeisu/model.py:510-544) of a training state dict:
    the 34 FoldedAEISU tensors as float32 numpy arrays."""
    s = _arrays(state)
    out = {}
    for name, cin, cout, k in CONVOLUTIONS:
        out[f"{name}.weight"] = s[f"{name}.weight"] + _conv_addition(s, name, cin, cout, k)
        out[f"{name}.bias"] = s[f"{name}.bias"]
    out["analysis_rgb_basis"] = (s["analysis_rgb_basis"] + np.diag(s["analysis_rgb_basis_diag"])
                                 + s["analysis_rgb_basis_u"] @ s["analysis_rgb_basis_v"])
    out["analysis_rgb_mix"] = (s["analysis_rgb_mix"] + s["analysis_rgb_mix_bt709_gain"] * np.array(BT709)
                               + s["analysis_rgb_mix_uniform_gain"] * np.full(3, 1.0 / 3.0))
    for key, short, seed in STENCILS:
        out[f"analysis_{key}"] = (s[f"analysis_{key}"] + s[f"analysis_{short}_seed_gain"] * np.array(seed)
                                  + s[f"analysis_{short}_curve_gain"] * np.array(CURVE))
    dense = np.einsum("j,jtp->tp", s["base_rep_slopes"], s["base_rep_kernels"])
    out["base_kernel"] = s["base_kernel"] + dense + _structured_base(s).reshape(4, 25).T
    mixed = np.einsum("mk,mphw->kphw", s["basis_mix_matrix"], _basis_bank(s))
    out["basis_raw"] = s["basis_raw"] + mixed.reshape(16, 4, 25)
    return {k: np.ascontiguousarray(v, np.float32) for k, v in out.items()}

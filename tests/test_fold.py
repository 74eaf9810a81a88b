"""Training checkpoints: folding their training-only coordinates into the deployed tensors, as
the reference's load_model does (aeisu/runtime.py:49-52, fold_model of aeisu/model.py:599-602).

tests/golden/training_checkpoint.npz holds the reference's own folded tensors and upscale
output for a seeded training state (make_golden.py, section "training"); the state itself is
regenerated here from the same seeds."""
import numpy as np
import pytest

from conftest import GOLDEN
from oracle import aeisu_np as O
from aeisu_b200 import fold
from aeisu_b200.runtime import flatten_folded
from aeisu_b200.synthetic import make_frame, random_folded_state, seeded_training_state


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "training_checkpoint.npz")


def training_state(g):
    state = seeded_training_state(random_folded_state(int(g["weight_seed"])), int(g["branch_seed"]),
                                  float(g["branch_std"]))
    assert list(state) == [str(k) for k in g["keys"]], "training layout differs from the reference's"
    return state


def test_fold_matches_the_reference(golden):
    folded = fold.fold_training_state(training_state(golden))
    assert sorted(folded) == sorted(str(k) for k in golden["folded_keys"])
    for key, value in folded.items():
        ref = golden[f"folded.{key}"]
        assert value.shape == ref.shape and value.dtype == np.float32, key
        scale = max(float(np.abs(ref).max()), 1e-30)
        assert float(np.abs(value - ref).max()) <= 2e-6 * scale, key
    # the fold changes every deployed tensor (the branches are active), so the check has teeth
    base = random_folded_state(int(golden["weight_seed"]))
    assert all(not np.array_equal(folded[k], base[k]) for k in folded if not k.endswith(".bias"))
    flatten_folded(folded)   # the C ABI's 34-tensor layout accepts it


def test_folded_model_output_matches_the_reference(golden):
    folded = fold.fold_training_state(training_state(golden))
    frame = make_frame(int(golden["frame_seed"]), int(golden["h"]), int(golden["w"]))
    assert np.array_equal(frame, golden["frame"])
    out = O.upscale(O.FoldedModel(folded), O.u8_to_chw(frame), 0)
    assert float(np.abs(out - golden["upscale_f32"]).max()) <= 2e-6


def test_training_state_is_detected_and_checked_strictly(golden):
    state = training_state(golden)
    assert fold.is_training_state(state)
    assert not fold.is_training_state(random_folded_state(1))
    missing = dict(state)
    del missing["basis_mix_matrix"]
    with pytest.raises(ValueError, match="missing"):
        fold.fold_training_state(missing)
    extra = dict(state, stray=np.zeros(1, np.float32))
    with pytest.raises(ValueError, match="unexpected"):
        fold.fold_training_state(extra)
    bad = dict(state)
    bad["refine_540.rep_row"] = np.zeros((64, 32, 3, 1), np.float32)
    with pytest.raises(ValueError, match="shape"):
        fold.fold_training_state(bad)


def test_templates_are_l1_normalised():
    for t in (fold.directional_templates(), fold.structural_5x5_templates()):
        assert np.allclose(np.abs(t).sum(axis=(1, 2)), 1.0, atol=1e-6)
    ring = fold.outer_ring_templates()
    assert ring.shape == (16, 5, 5) and ring.sum() == 16 and ring[:, 1:4, 1:4].sum() == 0

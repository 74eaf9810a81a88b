"""aeisu_upscale_u8_noalloc: the allocation-free device-I/O upscale, for hosts that cannot
allocate GPU memory when they submit frames (see include/aeisu.h).

Its output must match the regular aeisu_upscale_u8 entry point on the same device buffers,
call after call, even though every call reuses the same static scratch array.  This file is
collected last on purpose, so a run that stops at the first failure has already run every
other test; it also passes when run alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

from aeisu_b200 import Model, _lib
from aeisu_b200.synthetic import make_frames, random_folded_state

pytestmark = pytest.mark.gpu


def u8_close(a, b):
    diff = np.abs(a.astype(int) - b.astype(int))
    return diff.max() <= 1 and (diff > 0).mean() <= 1e-3


def run_both(model, frames):
    import torch
    lib = _lib.lib()
    src = torch.from_numpy(frames).cuda()
    n, h, w, _ = frames.shape
    regular = torch.empty((n, 2 * h, 2 * w, 3), dtype=torch.uint8, device="cuda")
    noalloc = torch.full((n, 2 * h, 2 * w, 3), 7, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.aeisu_upscale_u8(model._handle(), src.data_ptr(), n, h, w, 0, regular.data_ptr(),
                                    _lib.IO_DEVICE, stream))
    _lib.check(lib.aeisu_upscale_u8_noalloc(model._handle(), src.data_ptr(), n, h, w, noalloc.data_ptr(), stream))
    model.synchronize(stream, 60000.0)
    torch.cuda.synchronize()
    return regular.cpu().numpy(), noalloc.cpu().numpy()


@pytest.mark.parametrize("precision", ["fp32", "fp16", "mixed"])
def test_noalloc_matches_regular_entry_point_twice(precision):
    if precision == "mixed":
        from spyr8_helpers import build_artifact
        state = random_folded_state(41, coeff_gain=0.5)
        model = Model.from_spyr8_bytes(build_artifact(state, make_frames(600, 2, 64, 96)), "cuda:0", "mixed")
    else:
        model = Model.from_folded_state(random_folded_state(12), "cuda:0", precision)
    try:
        # two calls in a row on different content: the shared scratch keeps the previous call's
        # data, which must not leak into the next result
        for seed, shape in ((70, (2, 72, 100)), (90, (3, 41, 67))):
            frames = make_frames(seed, *shape)
            regular, noalloc = run_both(model, frames)
            assert u8_close(regular, noalloc), f"{precision}: no-allocation output differs (seed {seed})"
    finally:
        model.close()


def test_noalloc_rejects_frames_beyond_its_scratch():
    import torch
    model = Model.from_folded_state(random_folded_state(12), "cuda:0", "fp16")
    try:
        lib = _lib.lib()
        src = torch.zeros((1, 1080, 1920, 3), dtype=torch.uint8, device="cuda")
        dst = torch.zeros((1, 2160, 3840, 3), dtype=torch.uint8, device="cuda")
        status = lib.aeisu_upscale_u8_noalloc(model._handle(), src.data_ptr(), 1, 1080, 1920, dst.data_ptr(), None)
        assert status == _lib.INVALID_ARG and "scratch" in _lib.last_error()
        # the handle keeps working afterwards
        regular, noalloc = run_both(model, make_frames(5, 1, 40, 40))
        assert u8_close(regular, noalloc)
    finally:
        model.close()

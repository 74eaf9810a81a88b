"""aeisu_upscale_u8_noalloc: the allocation-free device-I/O upscale, for hosts that cannot
allocate GPU memory when they submit frames (see include/aeisu.h).

Its output must equal the regular aeisu_upscale_u8 entry point's on the same device buffers,
byte for byte (the same kernels run on the same inputs), call after call, even though every
call reuses the same static scratch array.  This file is collected last on purpose, so a run
that stops at the first failure has already run every other test; it also passes when run
alone in a fresh process."""
import numpy as np
import pytest

from aeisu_b200 import Model, _lib
from aeisu_b200.runtime import CUDA_STREAM_LEGACY
from aeisu_b200.synthetic import make_frames, random_folded_state

pytestmark = pytest.mark.gpu


def run_both(model, frames):
    """Both entry points on the same device frames, on torch's current stream.  torch's default
    stream is the legacy stream (handle 0), which the C ABI reads as "the handle's own stream"
    (non-blocking, unordered with legacy-stream work): pass cudaStreamLegacy instead, so that
    the sentinel fill below is ordered before both calls."""
    import torch
    lib = _lib.lib()
    src = torch.from_numpy(frames).cuda()
    n, h, w, _ = frames.shape
    regular = torch.empty((n, 2 * h, 2 * w, 3), dtype=torch.uint8, device="cuda")
    noalloc = torch.full((n, 2 * h, 2 * w, 3), 7, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream or CUDA_STREAM_LEGACY
    _lib.check(lib.aeisu_upscale_u8(model._handle(), src.data_ptr(), n, h, w, 0, regular.data_ptr(),
                                    _lib.IO_DEVICE, stream))
    _lib.check(lib.aeisu_upscale_u8_noalloc(model._handle(), src.data_ptr(), n, h, w, noalloc.data_ptr(), stream))
    model.synchronize(stream, 60000.0)
    torch.cuda.synchronize()
    return regular.cpu().numpy(), noalloc.cpu().numpy()


def open_model(precision):
    if precision == "mixed":
        from spyr8_helpers import build_artifact
        state = random_folded_state(41, coeff_gain=0.5)
        return Model.from_spyr8_bytes(build_artifact(state, make_frames(600, 2, 64, 96)), "cuda:0", "mixed")
    return Model.from_folded_state(random_folded_state(12), "cuda:0", precision)


@pytest.mark.parametrize("precision", ["fp32", "fp16", "mixed"])
def test_noalloc_matches_regular_entry_point_twice(precision):
    model = open_model(precision)
    try:
        # two calls in a row on different content: the shared scratch keeps the previous call's
        # data, which must not leak into the next result
        for seed, shape in ((70, (2, 72, 100)), (90, (3, 41, 67))):
            frames = make_frames(seed, *shape)
            regular, noalloc = run_both(model, frames)
            np.testing.assert_array_equal(noalloc, regular, err_msg=f"{precision}: seed {seed}")
    finally:
        model.close()


# Batches that do not fit the scratch array at once run in chunks of whole frames, each chunk
# rewriting the region table and reusing the same activation memory.  512 x 512 frames (padded
# 544 x 544) fit two at a time on the mixed and FP16 routes and one at a time on FP32, so these
# batches take two chunks, the last one partial.
@pytest.mark.parametrize("precision,n", [("mixed", 3), ("fp16", 3), ("fp32", 2)])
def test_noalloc_batch_in_several_chunks(precision, n):
    model = open_model(precision)
    try:
        for seed in (71, 72):
            frames = make_frames(seed, n, 512, 512)
            regular, noalloc = run_both(model, frames)
            np.testing.assert_array_equal(noalloc, regular, err_msg=f"{precision}: seed {seed}")
    finally:
        model.close()


# Per padded input pixel the scratch holds about 80 bytes on the mixed route, 96 on FP16 and
# 224 on FP32, so the largest frames are about 0.83, 0.69 and 0.29 Mpixel of padded input.
@pytest.mark.parametrize("precision,h,w", [("fp16", 1080, 1920), ("mixed", 1080, 1920), ("fp32", 540, 960)])
def test_noalloc_rejects_frames_beyond_its_scratch(precision, h, w):
    import torch
    model = open_model(precision)
    try:
        lib = _lib.lib()
        src = torch.zeros((1, h, w, 3), dtype=torch.uint8, device="cuda")
        dst = torch.zeros((1, 2 * h, 2 * w, 3), dtype=torch.uint8, device="cuda")
        status = lib.aeisu_upscale_u8_noalloc(model._handle(), src.data_ptr(), 1, h, w, dst.data_ptr(), None)
        assert status == _lib.INVALID_ARG and "scratch" in _lib.last_error()
        # the handle keeps working afterwards
        regular, noalloc = run_both(model, make_frames(5, 1, 40, 40))
        np.testing.assert_array_equal(noalloc, regular)
    finally:
        model.close()

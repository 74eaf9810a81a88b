"""Sibling handles (aeisu_open_sibling; CudaRuntime::CreateSibling,
optimized/native/src/neural/srcpyr/SrcPyrCudaRuntime.cu:5392-5402): one copy of the device
weights, a stream and workspace per handle."""
import threading

import numpy as np
import pytest

from conftest import staged
from aeisu_b200 import Model, load_model
from aeisu_b200.synthetic import make_frames, random_folded_state

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("precision", ["fp32", "mixed"])
def test_sibling_matches_its_parent_and_outlives_it(precision):
    if precision == "mixed":
        parent = load_model(staged("adaptive_fp8.bin"), "cuda:0", "mixed")
    else:
        parent = Model.from_folded_state(random_folded_state(12), "cuda:0", "fp32")
    child = parent.sibling()
    try:
        assert "sibling" in child.report and child.precision == parent.precision
        frames = make_frames(1500, 3, 72, 100)
        expected = parent.upscale_u8(frames, 0)
        np.testing.assert_array_equal(child.upscale_u8(frames, 0), expected)
        np.testing.assert_array_equal(child.upscale_u8(frames, 32), parent.upscale_u8(frames, 32))
        parent.close()   # the shared weights stay alive while a sibling holds them
        np.testing.assert_array_equal(child.upscale_u8(frames, 0), expected)
        grandchild = child.sibling()
        child.close()
        np.testing.assert_array_equal(grandchild.upscale_u8(frames, 0), expected)
        grandchild.close()
    finally:
        parent.close()
        child.close()


def test_siblings_run_concurrently_on_their_own_threads():
    """Two siblings, one host thread each, device I/O on their own streams at the same time: each
    gets exactly the single-handle result, every time."""
    import torch
    parent = load_model(staged("adaptive_fp8.bin"), "cuda:0", "mixed")
    handles = [parent, parent.sibling()]
    try:
        batches = [make_frames(1600 + k, 4, 96, 160) for k in range(2)]
        expected = [parent.upscale_u8(b, 0) for b in batches]
        results = [[], []]

        def worker(k):
            stream = torch.cuda.Stream()
            src = torch.from_numpy(batches[k]).cuda()
            with torch.cuda.stream(stream):
                for _ in range(4):
                    out = handles[k].upscale_u8(src, 0)
                    stream.synchronize()
                    results[k].append(out.cpu().numpy())
        threads = [threading.Thread(target=worker, args=(k,)) for k in range(2)]
        for th in threads:
            th.start()
        for th in threads:
            th.join()
        for k in range(2):
            assert len(results[k]) == 4
            for got in results[k]:
                np.testing.assert_array_equal(got, expected[k])
    finally:
        for h in handles:
            h.close()


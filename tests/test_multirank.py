"""The multi-GPU host logic of bench.py on CPU, as two gloo ranks: the timing rule (every rank
reports the slowest rank's time), distinct frames per rank (frame-parallel ranks share no work)
and the whole-job output count (frame-parallel: every rank's batch; row bands: one frame)."""
import os
import socket
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir):
    sys.path.insert(0, str(ROOT))
    import hashlib
    import torch.distributed as dist
    import bench
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        slowest = bench.max_over_ranks(1.5 + rank, dist, "cpu")
        frames = bench.gen_frames(bench.rank_seed(rank), 2, 32, 48, "area")
        digests = [None] * world
        dist.all_gather_object(digests, hashlib.sha256(frames.tobytes()).hexdigest())
        Path(out_dir, f"rank{rank}.txt").write_text(f"{slowest} {len(set(digests))}")
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        slowest, distinct = (tmp_path / f"rank{r}.txt").read_text().split()
        assert float(slowest) == 1.5 + world - 1     # the slowest rank's time on every rank
        assert int(distinct) == world                # no two ranks upscale the same frames


@pytest.mark.parametrize("world", [1, 2, 8])
def test_whole_job_output_pixels(world):
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.output_pixels(720, 1280, 64, world, band=False) == 4 * 720 * 1280 * 64 * world
    assert bench.output_pixels(4320, 7680, 1, world, band=True) == 4 * 4320 * 7680

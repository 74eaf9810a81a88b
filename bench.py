"""Benchmark: 2x output Mpix/s of the AEISU inference path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload mixed720|fp16_1080|tiled1080|stream4k] [--precision P]

One step = one pass of the path over one batch of synthetic frames (default workload
"mixed720": 64 frames of 1280x720 uint8 RGB -> 2560x1440, FP8/FP16 mixed weights of the
SPYR8 artifact, full frame).  Multi-GPU: one process per GPU (torchrun); every rank
upscales its own batch (frame-parallel, weak scaling, no data-path collective); timing is
CUDA events with barriers, max over ranks.  Prints one JSON line on rank 0.

`value` times the device-resident path (inputs already in HBM; inputs+outputs are larger
than L2, so no flush is needed).  `e2e` times the same batch through the public C ABI with
pinned host buffers (allocated on the GPU's NUMA node): host->device copy, compute,
device->host copy inside the region, beside the host link's ceiling for the same bytes.
`roofline` holds the dominant stage against its bound and `roofline.step` the whole step
against the north-star roofline, max(controller FLOPs at tensor peak, head bytes at HBM
bandwidth), with the E4M3 rate measured in the run by a tcgen05 probe.  The default workload
also records configuration 5 at this N (`stream4k`, `band8k`) and the 1080p latency over 1000
distinct frames, device-resident and end to end.  `--impl reference` times the reference
algorithm's CPU implementation (the numpy port in oracle/, FP32) on the host cores with the
same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
WEIGHTS = ROOT / "oracle" / "_ref" / "weights"

WORKLOADS = {
    # name: (frames per step, h, w, tile, precision, checkpoint, degradation, metric-config)
    "mixed720": (64, 720, 1280, 0, "mixed", "adaptive_fp8.bin", "area"),
    "fp16_1080": (1, 1080, 1920, 0, "fp16", "aeisu_area.pt", "area"),
    "mixed1080": (1, 1080, 1920, 0, "mixed", "adaptive_fp8.bin", "area"),
    "tiled1080": (32, 1080, 1920, 256, "fp16", "aeisu_bicubic.pt", "bicubic"),
    "stream4k": (8, 2160, 3840, 0, "mixed", "adaptive_fp8.bin", "area"),
    # the conventional-CUDA INT8/FP16 deployment's artifact (optimized/shader/weights)
    "int8_720": (64, 720, 1280, 0, "int8", "aeisu_int8_fp16.pt", "area"),
    "int8_1080": (1, 1080, 1920, 0, "int8", "aeisu_int8_fp16.pt", "area"),
    # one 7680x4320 input frame split into one row band per GPU (strong scaling)
    "band8k": (1, 4320, 7680, 0, "mixed", "adaptive_fp8.bin", "area"),
}
BAND_WORKLOADS = {"band8k"}
# controller FLOPs per padded LR pixel (paper MAC table: 11,520 MAC) and head bytes per LR pixel
CONTROLLER_FLOP_PER_PX = 2 * 11520
HEAD_BYTES_PER_PX = 3 + 32 + 12
# controller MACs per padded LR pixel by arithmetic on the mixed route: f16 project 256 +
# refine 4,608 + head 1,024; e4m3 compress 512 + bottlenecks 4,608 + expand 512
MIXED_F16_MACS, MIXED_E4M3_MACS = 5888, 5632
# DRAM bytes (read + write) of one launch of the dominant kernel on the default workload, from
# one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum); reported as roofline.traffic
# with its source, since a run cannot read DRAM counters itself
RECORDED_TRAFFIC = {"mixed720": ("reconstruction_ms", 2.075e9 + 0.687e9,
                                 "ncu capture of one k_tc_head<1, true, true> launch (TMA coefficient "
                                 "rows), 64 x 1280x720 mixed")}


def padded(h, w):
    return h + 32 + (-h % 32), w + 32 + (-w % 32)


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def rank_seed(rank):
    """Frame seed of a rank: every rank upscales its own distinct frames (frame-parallel)."""
    return 10_000 * (rank + 1)


def output_pixels(h, w, frames_per_rank, world, band):
    """2x output pixels one step produces over the whole job: frame-parallel ranks each upscale
    their own batch; row-band ranks share one frame (each writes its own rows)."""
    return 4 * h * w * frames_per_rank * (1 if band else world)


def max_over_ranks(x, dist, device):
    """The slowest rank's value: multi-GPU times are the maximum over ranks."""
    import torch
    t = torch.tensor([float(x)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gen_frames(seed, count, h, w, degradation):
    """Distinct seeded frames, rendered in a spawn pool (before any CUDA use)."""
    from aeisu_b200.synthetic import make_frame
    import multiprocessing as mp
    procs = max(1, min(count, (os.cpu_count() or 2) // max(1, dist_env()[2]) - 1, 32))
    args = [(seed + i, h, w, degradation) for i in range(count)]
    if procs == 1:
        return np.stack([make_frame(*a) for a in args])
    with mp.get_context("spawn").Pool(procs) as pool:
        return np.stack(pool.starmap(make_frame, args))


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons of the benchmarked GPU, sampled during the
    timed region: NVML every ~10 ms (the timed region can be under 100 ms), else nvidia-smi."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    # NVML clock-event reason bits (nvml.h: SwPowerCap 0x4, HwSlowdown 0x8, SwThermal 0x20, HwThermal 0x40)
    BITS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, device_index, period=0.01):
        self.device_index = device_index
        self.period = period
        self.proc = None
        self.thread = None
        self.stop = threading.Event()
        self.lines = []     # nvidia-smi csv lines
        self.samples = []   # NVML (sm_mhz, max_mhz, reason bits)

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:   # the CUDA device's own NVML handle (CUDA and NVML indices can differ)
            import torch
            uuid = str(torch.cuda.get_device_properties(self.device_index).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.device_index)

    def _poll(self, nvml, handle):
        while not self.stop.is_set():
            try:
                sm = nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM)
                mx = nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM)
                bits = nvml.nvmlDeviceGetCurrentClocksThrottleReasons(handle)
                self.samples.append((float(sm), float(mx), int(bits)))
            except Exception:
                return
            self.stop.wait(self.period)

    def __enter__(self):
        try:
            nvml, handle = self._nvml_handle()
            self.thread = threading.Thread(target=self._poll, args=(nvml, handle), daemon=True)
            self.thread.start()
            return self
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.device_index), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        self.stop.set()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        elif self.thread:
            self.thread.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], [], set()
        for s_mhz, m_mhz, bits in self.samples:
            sm.append(s_mhz)
            mx.append(m_mhz)
            reasons.update(n for n in self.NAMES if bits & self.BITS[n])
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(self.NAMES, parts[4:8]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvml" if self.samples else "nvidia-smi"}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def tensor_probe(device_index):
    """Dense tcgen05 throughput of this GPU (aeisu_tensor_peak): kind::f16 and kind::f8f6f4 with
    E4M3 operands, M = 128, N = 256, two CTAs per SM, best of 5 launches of 4,096 MMAs each."""
    import ctypes as C
    from aeisu_b200 import _lib
    out = {}
    for name, kind in (("f16_tflops", 0), ("e4m3_tflops", 1)):
        v = C.c_double()
        _lib.check(_lib.lib().aeisu_tensor_peak(device_index, kind, 2, 4096, 5, C.byref(v)))
        out[name] = v.value
    out["how"] = "tcgen05.mma M=128 N=256, 296 CTAs x 4096 MMAs, one thread each, best of 5 launches"
    return out


def bind_to_gpu_numa(device_index):
    """Restrict this process to the host CPUs NVML lists as closest to the GPU (its NUMA node),
    so that pinned host buffers allocated afterwards are first touched on that node."""
    try:
        import pynvml
        import torch
        p = torch.cuda.get_device_properties(device_index)
        pynvml.nvmlInit()
        handle = pynvml.nvmlDeviceGetHandleByPciBusId(f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0")
        words = pynvml.nvmlDeviceGetCpuAffinity(handle, ((os.cpu_count() or 64) + 63) // 64)
        cpus = {64 * i + b for i, word in enumerate(words) for b in range(64) if (word >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return "not bound: no CPU of the GPU's node is available to this process"
        os.sched_setaffinity(0, cpus)
        return f"{len(cpus)} CPUs of the GPU's NUMA node"
    except Exception as e:   # NVML absent or the query unsupported: leave the affinity as it is
        return f"not bound: {type(e).__name__}"


def host_link_ceiling(dev, d2h_bytes, h2d_bytes, dist, world, reps=3):
    """Bytes per second of one plain pinned D2H copy of d2h_bytes and one H2D copy of
    h2d_bytes, on their own streams at once, on every rank at once (max over ranks): the host
    link's ceiling for the end-to-end step's traffic."""
    import torch
    dsrc = torch.empty(d2h_bytes, dtype=torch.uint8, device=dev)
    ddst = torch.empty(h2d_bytes, dtype=torch.uint8, device=dev)
    hdst = torch.empty(d2h_bytes, dtype=torch.uint8).pin_memory()
    hsrc = torch.empty(h2d_bytes, dtype=torch.uint8).pin_memory()
    s_out, s_in = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    best = float("inf")
    for r in range(reps + 1):
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        with torch.cuda.stream(s_out):
            hdst.copy_(dsrc, non_blocking=True)
        with torch.cuda.stream(s_in):
            ddst.copy_(hsrc, non_blocking=True)
        s_out.synchronize()
        s_in.synchronize()
        dt = time.perf_counter() - t0
        if world > 1:
            dt = max_over_ranks(dt, dist, dev)
        if r > 0:
            best = min(best, dt)
    del dsrc, ddst, hdst, hsrc
    return (d2h_bytes + h2d_bytes) / best


def distinct_frames(dev, seed, scenes, count, h, w):
    """`count` distinct seeded frames on the device: `scenes` rendered procedural scenes, the
    first `scenes` frames as rendered, every later one a rendered scene circularly shifted by a
    seeded offset and flipped by seeded bits (the scene statistics of the recipe, without
    rendering every frame)."""
    import torch
    base = torch.from_numpy(gen_frames(seed, scenes, h, w, "area")).to(dev)
    rng = np.random.default_rng(seed + 999)
    out = torch.empty((count, h, w, 3), dtype=torch.uint8, device=dev)
    for i in range(count):
        f = base[i % scenes]
        if i >= scenes:
            dy, dx, flips = int(rng.integers(1, h)), int(rng.integers(1, w)), int(rng.integers(0, 4))
            f = torch.roll(f, (dy, dx), (0, 1))
            if flips & 1:
                f = f.flip(0)
            if flips & 2:
                f = f.flip(1)
        out[i] = f
    return out


def _oracle_model(ckpt):
    """The reference's FP32 CPU path for a workload's checkpoint.  The INT8 artifact was exported
    from aeisu_area.pt (its FP16 weights are that checkpoint's, rounded), and the reference's
    CPU path has no INT8 arithmetic, so its baseline is that checkpoint in FP32."""
    from oracle import aeisu_np as O
    if ckpt == "aeisu_int8_fp16.pt":
        ckpt = "aeisu_area.pt"
    path = WEIGHTS / ckpt
    if path.suffix == ".pt":
        return O.load_folded(path)
    from aeisu_b200 import spyr8
    st, basis = spyr8.folded_state_from_spyr8(spyr8.read_spyr8(path.read_bytes()))
    return O.FoldedModel(st, basis=basis)


def _cpu_frames(model, frames, tile, threads):
    """Upscale `frames` (uint8 NHWC) with the FP32 numpy port: one frame per host thread,
    one BLAS thread per frame (numpy releases the GIL in its kernels)."""
    from concurrent.futures import ThreadPoolExecutor
    from threadpoolctl import threadpool_limits
    from oracle import aeisu_np as O
    with threadpool_limits(limits=1), ThreadPoolExecutor(threads) as ex:
        list(ex.map(lambda f: O.upscale_u8(model, f, tile), frames))


def _cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def measure_latency(dev, runs, scenes=40):
    """Latency of one 1920x1080 -> 3840x2160 frame (FP16, mixed and INT8 routes) over `runs`
    distinct seeded frames (distinct_frames: `scenes` rendered scenes, the rest seeded shifts and
    flips of them), p50 and p99:
    * device: input resident in HBM, CUDA events around each call on the launching stream;
    * end to end: through the public API with pinned host buffers, each call copying its uint8
      frame in, upscaling and copying the uint8 result out before it returns (host clock)."""
    import torch
    from aeisu_b200 import load_model
    frames = distinct_frames(dev, 50_000, min(scenes, runs), runs, 1080, 1920)
    host_frames = frames.cpu().pin_memory()
    out = torch.empty((2160, 3840, 3), dtype=torch.uint8, device=dev)
    host_out = torch.empty((2160, 3840, 3), dtype=torch.uint8).pin_memory()

    def pct(ms):
        ms = sorted(ms)
        return {"p50_ms": ms[len(ms) // 2], "p99_ms": ms[min(len(ms) - 1, int(len(ms) * 0.99))]}
    res = {}
    for precision, ckpt in (("fp16", "aeisu_area.pt"), ("mixed", "adaptive_fp8.bin"), ("int8", "aeisu_int8_fp16.pt")):
        model = load_model(WEIGHTS / ckpt, f"cuda:{dev.index}", precision)
        stream = torch.cuda.Stream(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(runs)]
        with torch.cuda.stream(stream):
            for i in range(10):
                model.upscale_u8(frames[i % runs], 0, out=out)
            for i in range(runs):
                ev[i][0].record(stream)
                model.upscale_u8(frames[i], 0, out=out)
                ev[i][1].record(stream)
        torch.cuda.synchronize(dev)
        res[precision] = pct([a.elapsed_time(b) for a, b in ev])
        for i in range(10):
            model.upscale_u8(host_frames[i % runs], 0, out=host_out)
        wall = []
        for i in range(runs):
            t0 = time.perf_counter()
            model.upscale_u8(host_frames[i], 0, out=host_out)
            wall.append((time.perf_counter() - t0) * 1e3)
        res[precision]["e2e"] = pct(wall)
        model.close()
    res["config"] = (f"1920x1080 -> 3840x2160, batch 1, tile 0, {runs} distinct seeded frames "
                     f"({min(scenes, runs)} rendered scenes and seeded shifts/flips of them); device: input in HBM, "
                     "CUDA events per call on the launching stream; e2e: pinned host frame in, uint8 result in "
                     "pinned host memory on return (6,220,800 B H2D + 24,883,200 B D2H per call), host clock")
    return res


def measure_metrics(dev, out_u8, pairs, cpu_pairs=1):
    """Evaluation metrics (aeisu_distortion: encoded-Y MSE/PSNR + 11x11 Gaussian SSIM in FP64) on
    `pairs` float32 CHW pairs of the step's output size, device resident: CUDA events around
    batched calls on the launching stream; beside it the FP64 numpy port on `cpu_pairs` pair(s)."""
    import torch
    from aeisu_b200 import metrics
    from oracle import metrics_np as M
    m = min(pairs, out_u8.shape[0])
    target = out_u8[:m].permute(0, 3, 1, 2).float().div(255).contiguous()
    gen = torch.Generator(device=dev).manual_seed(7)
    pred = (target + 0.01 * torch.randn(target.shape, generator=gen, device=dev)).contiguous()
    _, _, H, W = target.shape
    stream = torch.cuda.Stream(dev)
    runs = 10
    with torch.cuda.stream(stream):
        for _ in range(3):
            metrics.distortion_batch(pred, target)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(runs):
            scores = metrics.distortion_batch(pred, target)
        end.record(stream)
    torch.cuda.synchronize(dev)
    ms = start.elapsed_time(end) / runs
    px = m * H * W
    hbm = measured_peaks()[0]
    nbytes = 2 * 3 * 4 * px
    p0, t0 = pred[0].cpu().numpy(), target[0].cpu().numpy()
    c0 = time.perf_counter()
    for _ in range(cpu_pairs):
        ref = M.distortion(p0, t0)
    cpu_s = (time.perf_counter() - c0) / cpu_pairs
    return {"value": px / (ms / 1e3) / 1e6, "unit": "pixel pairs Mpix/s", "ms_per_call": ms, "pairs_per_call": m,
            "frame": f"{W}x{H}", "dtype": "f32 in, f64 arithmetic",
            "hbm": {"achieved": nbytes / (ms / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                    "frac": nbytes / (ms / 1e3) / 1e9 / hbm},
            "fp64_flop_per_px": 284,
            "check_vs_port": {"y_ssim_abs_diff": abs(scores[0]["y_ssim"] - ref["y_ssim"]),
                              "y_mse_abs_diff": abs(scores[0]["y_mse"] - ref["y_mse"])},
            "cpu_port": {"value": H * W / cpu_s / 1e6, "unit": "pixel pairs Mpix/s", "cores": 1,
                         "kind": "port", "sample": f"{cpu_pairs} pair(s) {W}x{H}, numpy FP64"},
            "config": "the step's upscaled frames as targets, +N(0, 0.01) as predictions, crop 2, "
                      f"{runs} batched calls after 3 warm-up calls, inputs in HBM"}


def measure_png(out_u8, frames):
    """PNG egress (aeisu_png_encode): `frames` of the step's uint8 output, device resident, encoded
    per call into host memory (the D2H copy of the files is inside the timed region); beside it
    the reference's save_rgb encoder (PIL, zlib level 6) on one frame of the same output."""
    import io
    import torch
    from PIL import Image
    from aeisu_b200 import codec
    m = min(frames, out_u8.shape[0])
    x = out_u8[:m].contiguous()
    for _ in range(2):
        files = codec.encode_png(x)
    torch.cuda.synchronize(x.device)
    runs = 5
    t0 = time.perf_counter()
    for _ in range(runs):
        files = codec.encode_png(x)
    dt = (time.perf_counter() - t0) / runs
    _, H, W, _ = x.shape
    ours = sum(len(f) for f in files) / m
    frame = x[0].cpu().numpy()
    c0 = time.perf_counter()
    buf = io.BytesIO()
    Image.fromarray(frame).save(buf, format="PNG")
    pil_s = time.perf_counter() - c0
    return {"value": m * H * W / dt / 1e6, "unit": "Mpix/s encoded", "ms_per_call": dt * 1e3, "frames_per_call": m,
            "frame": f"{W}x{H}", "bytes_per_frame": ours, "raw_bytes_per_frame": H * W * 3,
            "pil_bytes_per_frame": len(buf.getvalue()),
            "cpu_reference": {"value": H * W / pil_s / 1e6, "unit": "Mpix/s encoded", "cores": 1,
                              "kind": "reference", "sample": f"PIL PNG save of 1 frame {W}x{H} (save_rgb's encoder)"},
            "config": "the step's uint8 output frames in HBM, files returned to host memory; wall clock over "
                      f"{runs} calls after 2 warm-up calls"}


def measure_png_ingress(frames_u8, count):
    """PNG ingress (aeisu_png_decode): `count` of the step's input frames, encoded by PIL as
    save_rgb writes them (zlib level 6), decoded per call from host memory (the upload inside the
    timed region) into a host array reused across calls (the download inside the timed region)
    and, beside it, into a CUDA tensor (frames left on the GPU for the upscaler); beside both
    read_rgb's decoder (PIL open + convert("RGB")) on a few of the same files, one core."""
    import io
    import torch
    from PIL import Image
    from aeisu_b200 import codec
    m = min(count, frames_u8.shape[0])
    files = []
    for i in range(m):
        buf = io.BytesIO()
        Image.fromarray(frames_u8[i]).save(buf, format="PNG")
        files.append(buf.getvalue())
    host = codec.decode_png(files)
    exact = bool(np.array_equal(host, frames_u8[:m]))
    dev = codec.decode_png(files, out="device")
    torch.cuda.synchronize()
    runs = 3
    t0 = time.perf_counter()
    for _ in range(runs):
        codec.decode_png(files, out=host)
    dt = (time.perf_counter() - t0) / runs
    t0 = time.perf_counter()
    for _ in range(runs):
        codec.decode_png(files, out=dev)
    torch.cuda.synchronize()
    dt_dev = (time.perf_counter() - t0) / runs
    _, H, W, _ = frames_u8.shape
    sample = min(4, m)
    c0 = time.perf_counter()
    for i in range(sample):
        with Image.open(io.BytesIO(files[i])) as im:
            np.asarray(im.convert("RGB"))
    pil_s = (time.perf_counter() - c0) / sample
    return {"value": m / dt, "unit": "frames/s decoded", "ms_per_call": dt * 1e3, "frames_per_call": m,
            "to_device": {"value": m / dt_dev, "unit": "frames/s decoded", "ms_per_call": dt_dev * 1e3},
            "frame": f"{W}x{H}", "bytes_per_file": sum(len(f) for f in files) / m, "pixels_equal_input": exact,
            "cpu_reference": {"value": 1.0 / pil_s, "unit": "frames/s decoded", "cores": 1, "kind": "reference",
                              "sample": f"PIL open + convert('RGB') of {sample} of the same files (read_rgb's decoder)"},
            "config": "PIL-written files (save_rgb's encoder, zlib level 6) in host memory, pixels into a host array "
                      f"reused across calls (to_device: into a CUDA tensor); wall clock over {runs} calls after 1 "
                      "warm-up call"}


def measure_train(dev, batch, sm_mhz=None):
    """Training reconstruction (aeisu_reconstruct_f32 + aeisu_reconstruct_backward_f32 through the
    autograd drop-in aeisu_b200.reconstruction.reconstruct) at the reference recipe's shape
    (configs/area.json: batch 32, 512x512 HR patches, source_pad 16 -> 288x288 sources, trim 32,
    basis_grad_stride 16): CUDA events around forward + backward on the launching stream, inputs
    in HBM (larger than L2).  Beside it the FP32 numpy port on one 288x288 sample."""
    import torch
    from aeisu_b200.reconstruction import reconstruct
    from oracle import reconstruct_np as R
    h = w = 288
    trim, stride = 32, 16
    ch, cw = h - trim, w - trim
    g = torch.Generator(device=dev).manual_seed(3)
    src = torch.rand((batch, 3, h, w), device=dev, generator=g)
    meta = (torch.randn((batch, 64, h // 2, w // 2), device=dev, generator=g) * 2).requires_grad_()
    base = (torch.randn((25, 4), device=dev, generator=g) * 0.05).requires_grad_()
    basis = (torch.randn((25, 16, 4), device=dev, generator=g) * 0.05).requires_grad_()
    grad = torch.randn((batch, 3, 2 * ch, 2 * cw), device=dev, generator=g)
    stream = torch.cuda.current_stream(dev)   # where a training loop runs its steps
    runs, warm = 10, 5
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3 * runs)]

    def zero_grad():   # optimizer.zero_grad(set_to_none=True), train.py:98
        meta.grad = base.grad = basis.grad = None

    for _ in range(warm):
        zero_grad()
        reconstruct(src, meta, base, basis, trim=trim, gradient_stride=stride).backward(grad)
    torch.cuda.synchronize(dev)
    for r in range(runs):
        zero_grad()
        ev[3 * r].record(stream)
        out = reconstruct(src, meta, base, basis, trim=trim, gradient_stride=stride)
        ev[3 * r + 1].record(stream)
        out.backward(grad)
        ev[3 * r + 2].record(stream)
    torch.cuda.synchronize(dev)
    # medians over the steps: autograd enqueues the backward from its worker thread, so one
    # step's interval can include a host-side stall (GIL) during which the GPU idles
    fwd = statistics.median(ev[3 * r].elapsed_time(ev[3 * r + 1]) for r in range(runs))
    bwd = statistics.median(ev[3 * r + 1].elapsed_time(ev[3 * r + 2]) for r in range(runs))
    px = batch * ch * cw
    sel = batch * ((ch + stride - 1) // stride) * ((cw + stride - 1) // stride)
    # FP32 FLOPs: filter assembly 2 x 1,600 + apply 2 x 300 per core pixel forward; filter
    # gradient 2 x 300 + coefficient gradient 2 x 1,600 backward; 2 x 1,700 per sampled pixel
    f_fwd, f_bwd = 3800.0 * px, 3800.0 * px + 3400.0 * sel
    mhz = sm_mhz or 1965.0
    peak = 148 * 128 * 2 * mhz * 1e6 / 1e12   # FP32 FMA pipe: 128 lanes per SM per clock
    c0 = time.perf_counter()
    s0 = src[:1].cpu().numpy()
    m0 = meta[:1].detach().cpu().numpy()
    b0, k0 = base.detach().cpu().numpy(), basis.detach().cpu().numpy()
    R.reconstruct(s0, m0, b0, k0, trim)
    R.reconstruct_backward(s0, m0, b0, k0, grad[:1].cpu().numpy(), trim, stride, 0)
    cpu_s = time.perf_counter() - c0
    total = fwd + bwd
    return {"value": 4 * px / (total / 1e3) / 1e6, "unit": "output Mpix/s (forward + backward)",
            "ms_per_step": total, "forward_ms": fwd, "backward_ms": bwd,
            "fp32": {"bound": "fp32 pipe", "forward_tflops": f_fwd / (fwd / 1e3) / 1e12,
                     "backward_tflops": f_bwd / (bwd / 1e3) / 1e12, "peak": peak, "unit": "TFLOP/s",
                     "forward_frac": f_fwd / (fwd / 1e3) / 1e12 / peak,
                     "backward_frac": f_bwd / (bwd / 1e3) / 1e12 / peak,
                     "peak_kind": f"nominal FP32 FMA rate at {mhz:.0f} MHz (148 SMs x 128 lanes)"},
            "cpu_port": {"value": 4 * ch * cw / cpu_s / 1e6, "unit": "output Mpix/s (forward + backward)",
                         "cores": 1, "kind": "port", "sample": f"1 source {w}x{h}, trim {trim}, stride {stride}, numpy FP32"},
            "config": f"batch {batch} x 3x{h}x{w} float32 sources, trim {trim} -> {2 * cw}x{2 * ch} outputs, "
                      f"gradient_stride {stride}, phase 0; medians of {runs} steps after {warm} warm-up steps, grads "
                      "set to None before each step, CUDA events on the current stream"}


def measure_config5(dev, dist, rank, world, barrier, stream_frames=512, batch=8, band_reps=5):
    """Config 5 of the benchmark set at this job's N, on the mixed route:
    * stream4k: a 512-frame stream of 3840x2160 frames split frame-parallel (512/N frames per
      rank, calls of 8 frames, distinct seeded frames per rank);
    * band8k: one 7680x4320 input frame (a 4K scene mirrored 2x2), one row band per rank.
    Each with inputs resident in HBM (CUDA events) and end to end through the public API with
    pinned host buffers (host clock); the slowest rank's time, whole-job output pixels."""
    import torch
    from aeisu_b200 import load_model
    model = load_model(WEIGHTS / "adaptive_fp8.bin", f"cuda:{dev.index}", "mixed")
    stream = torch.cuda.Stream(dev)
    h, w = 2160, 3840
    per_rank = stream_frames // world
    frames = distinct_frames(dev, 70_000 + 1000 * rank, 4, per_rank, h, w)
    outs = [torch.empty((batch, 2 * h, 2 * w, 3), dtype=torch.uint8, device=dev) for _ in range(2)]
    calls = [(i, min(batch, per_rank - i)) for i in range(0, per_rank, batch)]

    def timed(fn, reps=1):
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
        barrier()
        ms = e0.elapsed_time(e1) / reps
        return max_over_ranks(ms, dist, dev) if world > 1 else ms

    def wall(fn, reps=1):
        barrier()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        dt = (time.perf_counter() - t0) / reps
        return max_over_ranks(dt, dist, dev) if world > 1 else dt

    def run_stream():
        for k, (i, b) in enumerate(calls):
            model.upscale_u8(frames[i:i + b], 0, out=outs[k & 1][:b])
    with torch.cuda.stream(stream):
        model.upscale_u8(frames[:batch], 0, out=outs[0][:min(batch, per_rank)])
    stream_ms = timed(run_stream)
    stream_px = 4 * h * w * per_rank * world
    pool_n = min(per_rank, 32)
    pool = frames[:pool_n].cpu().pin_memory()
    host_out = torch.empty((batch, 2 * h, 2 * w, 3), dtype=torch.uint8).pin_memory()

    def run_stream_e2e():
        for i, b in calls:
            j = i % pool_n if i % pool_n + b <= pool_n else 0
            model.upscale_u8(pool[j:j + b], 0, out=host_out[:b])
    stream_e2e_s = wall(run_stream_e2e)
    big = torch.cat([torch.cat([frames[0], frames[0].flip(1)], 1), torch.cat([frames[0].flip(0), frames[0].flip(0).flip(1)], 1)], 0)
    del frames, outs, pool, host_out
    big = big.contiguous()
    big_out = torch.zeros((2 * 4320, 2 * 7680, 3), dtype=torch.uint8, device=dev)
    with torch.cuda.stream(stream):
        model.upscale_u8_band(big, rank, world, out=big_out)
    band_ms = timed(lambda: model.upscale_u8_band(big, rank, world, out=big_out), band_reps)
    host_big = big.cpu().pin_memory()
    host_big_out = torch.zeros((2 * 4320, 2 * 7680, 3), dtype=torch.uint8).pin_memory()
    model.upscale_u8_band(host_big, rank, world, out=host_big_out)
    band_e2e_s = wall(lambda: model.upscale_u8_band(host_big, rank, world, out=host_big_out), band_reps)
    band_px = 4 * 4320 * 7680
    model.close()
    return {
        "stream4k": {"value": stream_px / (stream_ms / 1e3) / 1e6, "unit": "output Mpix/s", "ms": stream_ms,
                     "e2e": {"value": stream_px / stream_e2e_s / 1e6, "unit": "output Mpix/s",
                             "h2d_bytes": per_rank * h * w * 3, "d2h_bytes": per_rank * 4 * h * w * 3},
                     "scaling": "strong", "config": f"{stream_frames} frames 3840x2160 -> 7680x4320, mixed, "
                     f"{per_rank} per GPU in calls of {batch}; distinct seeded frames per rank (4 rendered scenes and "
                     f"seeded shifts/flips); e2e: frames cycled through {pool_n} pinned host frames per rank"},
        "band8k": {"value": band_px / (band_ms / 1e3) / 1e6, "unit": "output Mpix/s", "ms": band_ms,
                   "e2e": {"value": band_px / band_e2e_s / 1e6, "unit": "output Mpix/s"},
                   "scaling": "strong", "config": f"one 7680x4320 frame -> 15360x8640, mixed, {world} row band(s) of "
                   f"the padded grid with 32-row recomputed halos, one per GPU; mean of {band_reps} calls"},
    }


def cpu_baseline(frames_u8, ckpt, tile, seconds=12.0):
    """Time the reference algorithm's CPU implementation (the oracle port, FP32, all host
    threads) on a bounded sample of the workload's frames."""
    model = _oracle_model(ckpt)
    threads = _cpu_threads()
    batch = [frames_u8[i % len(frames_u8)] for i in range(threads)]
    _cpu_frames(model, batch[:1], tile, 1)  # warm-up
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        _cpu_frames(model, batch, tile, threads)
        done += len(batch)
    dt = time.perf_counter() - t0
    h, w = frames_u8.shape[1:3]
    return {"value": 4 * h * w * done / dt / 1e6, "unit": "output Mpix/s", "cores": threads, "kind": "port",
            "sample": f"{done} frames of {w}x{h} (tile={tile}), {threads} at a time, through the FP32 numpy "
                      f"port of aeisu.runtime.upscale, {dt:.1f} s"}


def arm_config(workload, wl, precision, world):
    """The `config` of a bench line: the same dict on both arms (the reference arm samples
    this workload; its sampling is stated in its cpu_baseline.sample)."""
    n, h, w, tile, _, ckpt, _ = wl
    band = workload in BAND_WORKLOADS
    return {"workload": workload, "frames_per_step_per_gpu": n, "frame": f"{w}x{h}",
            "output": f"{2 * w}x{2 * h}", "tile": tile, "precision": precision, "checkpoint": ckpt,
            "l2": "inputs+outputs per step exceed the 126 MB L2; no flush needed",
            "parallelism": (f"row bands x{world} (32-row halos recomputed, no exchange)" if band
                            else f"frame-parallel x{world}")}


def run_reference(args, wl):
    rank, _, world = dist_env()
    if rank != 0:
        return
    n, h, w, tile, precision, ckpt, deg = wl
    threads = _cpu_threads()
    frames = gen_frames(1000, min(n, threads), h, w, deg)
    model = _oracle_model(ckpt)
    batch = [frames[i % len(frames)] for i in range(threads)]
    for _ in range(args.warmup):
        _cpu_frames(model, batch[:1], tile, 1)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _cpu_frames(model, batch, tile, threads)
    dt = time.perf_counter() - t0
    value = 4 * h * w * threads * args.steps / dt / 1e6
    line = {
        "impl": "reference", "metric": "2x output Mpix/s per B200 (FP8 mixed) frame-parallel; whole-job aggregate",
        "value": value, "unit": "output Mpix/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong" if args.workload in BAND_WORKLOADS else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded procedural scenes, 2x2 area / bicubic degradation)",
        "config": arm_config(args.workload, wl, args.precision or precision, world),
        "cpu_baseline": {"value": value, "unit": "output Mpix/s", "cores": threads, "kind": "port",
                         "sample": f"{threads} of the workload's {n} frames of {w}x{h} per step (a bounded sample), "
                                   f"one per host thread, through the FP32 numpy port of aeisu.runtime.upscale "
                                   f"(the reference's CPU path has FP32 arithmetic only; within 3% of its torch "
                                   f"path on the build container), on rank 0 only"},
        "e2e": {"value": value, "unit": "output Mpix/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=tuple(WORKLOADS), default="mixed720")
    ap.add_argument("--precision", default=None, help="override the workload's precision")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--latency-runs", type=int, default=1000,
                    help="1080p->4K single-frame latency runs (0 disables)")
    ap.add_argument("--png-frames", type=int, default=8,
                    help="frames per call of the PNG egress measurement (0 disables)")
    ap.add_argument("--png-decode-frames", type=int, default=64,
                    help="files per call of the PNG ingress measurement (0 disables)")
    ap.add_argument("--metric-pairs", type=int, default=8,
                    help="image pairs per call of the evaluation-metrics measurement (0 disables)")
    ap.add_argument("--train-batch", type=int, default=32,
                    help="sources per step of the training-reconstruction measurement (0 disables)")
    ap.add_argument("--e2e-steps", type=int, default=20, help="steps of the end-to-end measurement")
    ap.add_argument("--no-config5", dest="config5", action="store_false",
                    help="skip the 4K-stream and 8K-band measurements of the default workload")
    ap.add_argument("--fused-head", action="store_true",
                    help="run the reconstruction inside the controller's last kernel (aeisu_set_fused_head)")
    args = ap.parse_args()
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference(args, wl)
    args.warmup = max(args.warmup, 3)
    n, h, w, tile, precision, ckpt, deg = wl
    precision = args.precision or precision
    rank, local_rank, world = dist_env()

    # host-side frame generation happens before any CUDA call (spawn pool)
    frames = gen_frames(rank_seed(rank), n, h, w, deg)
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(frames, ckpt, tile, args.cpu_seconds)

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))

    from aeisu_b200 import load_model
    model = load_model(WEIGHTS / ckpt, f"cuda:{local_rank}", precision)
    if args.fused_head:
        model.set_fused_head(True)
    stream = torch.cuda.Stream(dev)
    src = torch.from_numpy(frames).to(dev)
    out = torch.empty((n, 2 * h, 2 * w, 3), dtype=torch.uint8, device=dev)
    band = args.workload in BAND_WORKLOADS   # every rank computes its own row band of the frame

    def upscale(x, o):
        if band:
            model.upscale_u8_band(x[0], rank, world, out=o[0])
        else:
            model.upscale_u8(x, tile, out=o)

    def step():
        with torch.cuda.stream(stream):
            upscale(src, out)

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    barrier()
    # stage timings of one step (events recorded between kernels, not synchronising)
    model.set_detailed_timing(True)
    step()
    torch.cuda.synchronize(dev)
    stages = model.timings()
    model.set_detailed_timing(False)

    launches0 = model.kernel_launches
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        barrier()
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        barrier()
    launches = model.kernel_launches - launches0
    ms = start.elapsed_time(end)
    if world > 1:
        ms = max_over_ranks(ms, dist, dev)
    ms_per_step = ms / args.steps
    out_mpix = output_pixels(h, w, n, world, band)
    value = out_mpix / (ms_per_step / 1e3) / 1e6

    # detailed per-stage pass over the timed steps for the roofline (separate, same stream)
    model.set_detailed_timing(True)
    stage_sum = {}
    for _ in range(args.steps):
        step()
        torch.cuda.synchronize(dev)
        for k, v in model.timings().items():
            stage_sum[k] = stage_sum.get(k, 0.0) + v
    model.set_detailed_timing(False)
    stage_ms = {k: v / args.steps for k, v in stage_sum.items() if k.endswith("_ms")}

    probe = tensor_probe(local_rank)
    latency = measure_latency(dev, args.latency_runs) if (rank == 0 and args.latency_runs > 0) else None
    metric_line = (measure_metrics(dev, out, args.metric_pairs)
                   if (rank == 0 and args.metric_pairs > 0 and not band) else None)
    png_line = measure_png(out, args.png_frames) if (rank == 0 and args.png_frames > 0 and not band) else None
    png_in_line = (measure_png_ingress(frames, args.png_decode_frames)
                   if (rank == 0 and args.png_decode_frames > 0 and not band) else None)
    train_line = (measure_train(dev, args.train_batch, clocks.summary().get("sm_mhz"))
                  if (rank == 0 and args.train_batch > 0 and not band) else None)

    # end-to-end through the public API with pinned host buffers, allocated after binding the
    # process to the GPU's NUMA node
    numa = bind_to_gpu_numa(local_rank)
    share = 1.0 / world if band else 1.0   # a row-band rank moves about 1/N of the frame
    h2d_bytes, d2h_bytes = int(n * h * w * 3 * share), int(n * 4 * h * w * 3 * share)
    host_src = torch.from_numpy(frames).pin_memory()
    host_out = torch.empty((n, 2 * h, 2 * w, 3), dtype=torch.uint8).pin_memory()
    upscale(host_src, host_out)
    barrier()
    t0 = time.perf_counter()
    e2e_steps = max(args.e2e_steps, 2)
    for _ in range(e2e_steps):
        upscale(host_src, host_out)
    e2e_dt = time.perf_counter() - t0
    if world > 1:
        e2e_dt = max_over_ranks(e2e_dt, dist, dev)
    e2e_value = out_mpix * e2e_steps / e2e_dt / 1e6
    del host_src, host_out
    ceiling = host_link_ceiling(dev, d2h_bytes, h2d_bytes, dist, world)
    e2e_rate = (h2d_bytes + d2h_bytes) * e2e_steps / e2e_dt

    # the other box-scale configurations: a 512-frame 4K stream split across the ranks, and one
    # 7680x4320 frame in one row band per rank
    extra = {}
    if args.workload == "mixed720" and args.config5:
        del out, src
        extra = measure_config5(dev, dist, rank, world, barrier)

    # roofline of the dominant stage
    hbm, tf_burst, tf_sus, peak_kind = measured_peaks()
    e4m3_peak = probe["e4m3_tflops"]
    hp, wp = padded(h, w)
    stage_names = ["analysis_project_ms", "compress_core_ms", "expand_ms", "refine_tail_ms", "reconstruction_ms"]
    dom = max(stage_names, key=lambda k: stage_ms.get(k, 0.0))
    # per-stage MAC per padded LR pixel (aeisu/model.py CONVOLUTIONS x pixel rates)
    macs = {"analysis_project_ms": 256, "compress_core_ms": 512 + 4608, "expand_ms": 512,
            "refine_tail_ms": 4608 + 1024}
    e4m3_stages = {"compress_core_ms", "expand_ms"} if precision == "mixed" else set()
    if dom == "reconstruction_ms":
        algo = HEAD_BYTES_PER_PX * h * w * n * share
        achieved = algo / (stage_ms[dom] / 1e3) / 1e9
        rec = RECORDED_TRAFFIC.get(args.workload)
        recorded = rec and rec[0] == dom and not args.precision
        roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": rec[1] if recorded else None, "traffic_source": rec[2] if recorded else None,
                "algorithmic_bytes": algo, "stage": "reconstruction head",
                "kernel": "k_tc_head" if precision != "fp32" else "k_f32_head", "peak_kind": peak_kind}
    else:
        algo = 2 * macs[dom] * hp * wp * n * share
        achieved = algo / (stage_ms[dom] / 1e3) / 1e12
        fp8 = dom in e4m3_stages
        peak = e4m3_peak if fp8 else tf_burst
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": None, "stage": dom[:-3],
                "peak_kind": "e4m3 tcgen05 probe (this run)" if fp8 else peak_kind}
    # the whole step against the north-star roofline: max(controller FLOPs at tensor peak, head
    # bytes at HBM bandwidth); the mixed route's FP8 share at the E4M3 probe's rate
    pad_px = hp * wp * n * share
    if precision == "mixed":
        f16_flop, e4m3_flop = 2 * MIXED_F16_MACS * pad_px, 2 * MIXED_E4M3_MACS * pad_px
    else:
        f16_flop, e4m3_flop = CONTROLLER_FLOP_PER_PX * pad_px, 0.0
    t_ctrl = f16_flop / (tf_burst * 1e12) + e4m3_flop / (e4m3_peak * 1e12)
    head_bytes = HEAD_BYTES_PER_PX * h * w * n * share
    t_head = head_bytes / (hbm * 1e9)
    t_roof = max(t_ctrl, t_head)
    roof["step"] = {"controller_flop": f16_flop + e4m3_flop, "controller_f16_flop": f16_flop,
                    "controller_e4m3_flop": e4m3_flop, "head_bytes": head_bytes,
                    "t_controller_ms": t_ctrl * 1e3, "t_head_ms": t_head * 1e3, "t_roof_ms": t_roof * 1e3,
                    "ms_per_step": ms_per_step, "frac": t_roof * 1e3 / ms_per_step,
                    "peaks": {"hbm_gbs": hbm, "f16_tflops": tf_burst, "e4m3_tflops": e4m3_peak,
                              "f16_kind": f"cuBLAS bf16 burst ({peak_kind})", "e4m3_kind": "tcgen05 probe, this run"}}
    roof["tensor_probe"] = probe

    if rank == 0:
        line = {
            "metric": "2x output Mpix/s per B200 (FP8 mixed) frame-parallel; whole-job aggregate",
            "value": value, "unit": "output Mpix/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong" if band else "weak",
            "vs_baseline": None, "dtype": {"fp32": "f32", "fp16": "f16", "mixed": "e4m3+f16", "int8": "s8 codes as f16+f16"}[precision],
            "data": "synthetic (seeded procedural scenes, 2x2 area / bicubic degradation)",
            "config": arm_config(args.workload, wl, precision, world),
            "stage_ms": stage_ms,
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "output Mpix/s",
                    "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes, "steps": e2e_steps,
                    "host_bytes_per_s": e2e_rate, "host_link_ceiling_bytes_per_s": ceiling,
                    "host_link_frac": e2e_rate / ceiling, "numa": numa,
                    "ceiling_how": "one plain pinned D2H copy of the step's output bytes and one H2D copy of its "
                                   "input bytes, on two streams at once, on every rank at once (max over ranks), "
                                   "best of 3"},
            **extra,
            "gpu_launches": int(launches),
            "latency_1080p": latency,
            "evaluation_metrics": metric_line,
            "png_egress": png_line,
            "png_ingress": png_in_line,
            "reconstruct_train": train_line,
            "clocks": clocks.summary(),
            "report": model.report,
        }
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

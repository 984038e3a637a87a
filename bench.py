#!/usr/bin/env python
"""Throughput of the implicitly zero-padded real 2D FFT cross-correlation.

Workload (one "step"): a 4096 x 4096 float32 image (N(0,1), seed 0) given by
its precomputed, transposed spectrum (2049 x 4096 complex64, computed once,
untimed); a batch of 32 templates of 256 x 256 (N(0,1) times a soft circular
mask of radius 120 px, then zero-mean / unit-variance; seed 1 + rank); the
full 32 x 4096 x 4096 float32 correlation maps.  One process per GPU, every
rank correlates its own batch (weak scaling, no data-path collective).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl zipfft|reference]
    python bench.py --workload search [--stats]   (template-matching search)

Prints one JSON line on rank 0.  `value` times K steps with the inputs
resident in HBM; `e2e` times K steps through zipfft.padded_rconv2d.corr with
each step's templates copied from pinned host memory (on a side stream into
one of two device buffers, overlapping the previous step) and each template's
peak score (corr's `peaks=` output, folded in by the kernel that writes the
map) read back every step.  `--impl reference` times the reference's own
correctness path (torch.fft on the host CPU, mgiammar/zipFFT
tests/test_real_conv_2d.py:110-123) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "2D padded cross-corr/sec at 4096² img, 256² tmpl; % HBM roofline; 1/2/4/8 GPU"
UNIT = "corr/s"
H = W = 4096
TH = TW = 256
BATCH = 32
# Minimum bytes per correlation: fp32 template + c64 image spectrum + fp32 output.
ALG_BYTES = TH * TW * 4 + H * (W // 2 + 1) * 8 + H * W * 4  # 134,512,640
L2_NOTE = ("no L2 flush: every step writes and reads back 2.1 GB of intermediates and "
           "writes 2.1 GB of maps, through the 126 MB L2 (the 67 MB spectrum is read "
           "by all 32 templates of the step's one column launch)")
WORKLOAD = ("4096^2 f32 image (spectrum precomputed) x 32 soft-masked 256^2 f32 templates "
            "per GPU, full 4096^2 maps")


def soft_mask(n: int = TH, r_in: float = 112.0, r_out: float = 120.0) -> torch.Tensor:
    """1 inside r_in, raised cosine to 0 at r_out, centred at ((n-1)/2, (n-1)/2)."""
    c = (n - 1) / 2.0
    yy, xx = torch.meshgrid(torch.arange(n, dtype=torch.float64),
                            torch.arange(n, dtype=torch.float64), indexing="ij")
    r = torch.sqrt((yy - c) ** 2 + (xx - c) ** 2)
    m = torch.where(r <= r_in, torch.ones_like(r),
                    torch.where(r >= r_out, torch.zeros_like(r),
                                0.5 * (1 + torch.cos(math.pi * (r - r_in) / (r_out - r_in)))))
    return m.float()


def make_templates(n: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    t = torch.randn((n, TH, TW), generator=g) * soft_mask()[None]
    t = t - t.mean(dim=(1, 2), keepdim=True)
    return (t / t.std(dim=(1, 2), keepdim=True)).contiguous()


def make_image(seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn((H, W), generator=g)


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        loaded = [s for s in sm if smax and s > 0.3 * smax] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# distributed plumbing (one process per GPU; timing only, no data collectives)
# ---------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# The clock sampler polls every 200 ms; a 20-step window of the headline
# workload lasts ~50 ms.  The K-step window is therefore timed repeatedly,
# back to back, until the windows add up to MIN_TIMED_MS of load, and the
# median window is reported (each window is exactly K steps, bracketed by a
# barrier and a device synchronisation, max over ranks).
MIN_TIMED_MS = 2000.0


def timed_windows(run_window, stream, world, min_total_ms=MIN_TIMED_MS, max_windows=500):
    """Times run_window() (K steps) repeatedly until min_total_ms of device
    time has passed; returns the list of window milliseconds, each the max
    over ranks (so every rank takes the same number of windows)."""
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    windows: list[float] = []
    while True:
        torch.cuda.synchronize()
        barrier(world)
        ev0.record(stream)
        run_window()
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        windows.append(max_over_ranks(ev0.elapsed_time(ev1), world))
        if sum(windows) >= min_total_ms or len(windows) >= max_windows:
            return windows


def window_summary(windows: list[float]) -> dict:
    return {"count": len(windows), "ms_min": min(windows), "ms_median": statistics.median(windows),
            "ms_max": max(windows), "reported": "median window"}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's torch.fft path on the host cores
# ---------------------------------------------------------------------------
def cpu_reference_rate(min_seconds: float = 10.0, templates_per_sample: int = 2):
    from oracle import xcorr_oracle as O

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    image_fft = torch.fft.rfftn(make_image(0))
    tm = make_templates(templates_per_sample, 1)
    O.reference_torch_path(tm[:1], image_fft, H, W, True, True)  # warm the FFT plans
    n, t0 = 0, time.perf_counter()
    while True:
        O.reference_torch_path(tm, image_fft, H, W, True, True)
        n += templates_per_sample
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return n / el, cores, n, el


def run_reference_arm(args, world, rank):
    if rank != 0:
        return 0
    from oracle import xcorr_oracle as O

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    image_fft = torch.fft.rfftn(make_image(0))
    per_step = 2
    tm = make_templates(per_step, 1)
    for _ in range(args.warmup):
        O.reference_torch_path(tm, image_fft, H, W, True, True)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.reference_torch_path(tm, image_fft, H, W, True, True)
    el = time.perf_counter() - t0
    value = per_step * args.steps / el
    sample = (f"{per_step} of the 32 templates per step (4096^2 full maps), "
              f"torch.fft on {cores} host threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": WORKLOAD, "image": [H, W],
                                        "template": [TH, TW], "templates_per_step": per_step,
                                        "output": "full"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def cufft_torch_rate(spec_nat, tm_dev, steps=5, warmup=3):
    """The explicit-pad torch.fft (cuFFT) pipeline on the same GPU, for comparison."""
    import torch.nn.functional as F

    def step():
        pad = F.pad(tm_dev, (0, W - TW, 0, H - TH))
        f = torch.fft.rfft2(pad)
        return torch.fft.irfft2(spec_nat[None] * torch.conj(f), s=(H, W))

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        out = step()
    e.record()
    torch.cuda.synchronize()
    del out
    ms = s.elapsed_time(e) / steps
    return tm_dev.shape[0] / (ms / 1e3), ms


def image_spectrum_timing(image, steps=20, warmup=3):
    """The library's image-spectrum path (row + in-place column kernels) and
    torch.fft.rfftn + transpose (cuFFT) on the same image.  Image and spectrum
    together (134 MB at 4096^2) exceed L2, so repeated calls stream from HBM."""
    from zipfft_b200 import padded_rconv2d as P

    out = torch.empty((W // 2 + 1, H), dtype=torch.complex64, device=image.device)

    def ours():
        P.image_spectrum(image, out)

    def theirs():
        return torch.fft.rfftn(image).transpose(0, 1).contiguous()

    res = {}
    for name, fn in (("ms", ours), ("cufft_torch_ms", theirs)):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            fn()
        e.record()
        torch.cuda.synchronize()
        res[name] = s.elapsed_time(e) / steps
    alg = H * W * 4 + (W // 2 + 1) * H * 8
    res.update({"algorithmic_bytes": alg, "achieved_gbs": alg / (res["ms"] / 1e3) / 1e9,
                "launches": 2, "what": "zipfft.padded_rconv2d.image_spectrum of the 4096^2 "
                                      "image: (W/2+1, H) complex64 conv_data"})
    return res


# ---------------------------------------------------------------------------
# The other measurement configurations (N = 1, rank 0): throughput of each
# one through zipfft.padded_rconv2d.corr (and the search at the search
# configuration's shapes), with the template content each one specifies.
# ---------------------------------------------------------------------------
def unit_variance(t: torch.Tensor) -> torch.Tensor:
    t = t - t.mean(dim=(-2, -1), keepdim=True)
    return (t / t.std(dim=(-2, -1), keepdim=True)).contiguous()


def gaussian_blob_templates(n: int, size: int, sigma: float, noise_sd: float,
                            seed: int) -> torch.Tensor:
    """A Gaussian blob of width sigma centred in each template, plus
    N(0, noise_sd) noise, then zero mean and unit variance."""
    g = torch.Generator().manual_seed(seed)
    c = (size - 1) / 2.0
    ax = torch.arange(size, dtype=torch.float64)
    yy, xx = torch.meshgrid(ax, ax, indexing="ij")
    blob = torch.exp(-((yy - c) ** 2 + (xx - c) ** 2) / (2 * sigma ** 2)).float()
    return unit_variance(blob[None] + noise_sd * torch.randn((n, size, size), generator=g))


# (key, description, image size, template size, templates per call, content, timed calls)
OTHER_CONFIGS = [
    ("1", "1024^2 image N(0,1), 4 templates 128^2 N(0,1) zero-mean unit-variance, full maps",
     1024, 128, 4, "randn", 400),
    ("3", "4096^2 image N(0,1), 64 templates 512^2: Gaussian blob sigma 20 px + N(0, 0.1), "
          "zero-mean unit-variance, full maps", 4096, 512, 64, "blob", 5),
    ("4", "3840^2 image N(0,1), 128 templates 384^2 N(0,1) zero-mean unit-variance, full maps "
          "(radix-3/5 path)", 3840, 384, 128, "randn", 4),
]


def measure_configs(dev) -> dict:
    import zipfft
    from zipfft_b200 import padded_rconv2d as P

    peak, peak_src = measured_hbm_peak()
    res = {}
    for key, desc, n, h, b, kind, calls in OTHER_CONFIGS:
        g = torch.Generator().manual_seed(0)
        spec = P.image_spectrum(torch.randn((n, n), generator=g).to(dev))
        if kind == "blob":
            tm = gaussian_blob_templates(b, h, 20.0, 0.1, 1)
        else:
            tm = unit_variance(torch.randn((b, h, h), generator=torch.Generator().manual_seed(1)))
        tm = tm.to(dev)
        ws = torch.empty((b, n, n // 2 + 1), dtype=torch.complex64, device=dev)
        out = torch.empty((b, n, n), dtype=torch.float32, device=dev)
        for _ in range(3):
            zipfft.padded_rconv2d.corr(tm, ws, spec, out, n, n)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(calls):
            zipfft.padded_rconv2d.corr(tm, ws, spec, out, n, n)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / calls
        rate = b / (ms / 1e3)
        alg = h * h * 4 + n * (n // 2 + 1) * 8 + n * n * 4
        res[key] = {"workload": desc, "value": rate, "unit": UNIT, "ms_per_call": ms,
                    "calls": calls, "algorithmic_bytes_per_corr": alg,
                    "achieved_gbs": alg * rate / 1e9, "frac": alg * rate / 1e9 / peak,
                    "peak_source": peak_src}
        del spec, tm, ws, out
        torch.cuda.empty_cache()
    res["5"] = search_rate(dev, steps=2, warmup=1)
    return res


def run_gpu_arm(args, world, rank, local):
    import zipfft
    from zipfft_b200 import _lib

    BATCH = args.batch
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)

    image = make_image(0).to(dev)
    spec_nat = torch.fft.rfftn(image)                 # setup only (untimed)
    spec_T = spec_nat.transpose(0, 1).contiguous()    # (W/2+1, H) as the API expects
    tm_host = make_templates(BATCH, 1 + rank).pin_memory()
    tm = tm_host.to(dev)
    ws = torch.empty((BATCH, H, W // 2 + 1), dtype=torch.complex64, device=dev)
    out = torch.empty((BATCH, H, W), dtype=torch.float32, device=dev)

    def step():
        zipfft.padded_rconv2d.corr(tm, ws, spec_T, out, H, W)

    # ---- device-resident throughput --------------------------------------
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    host_s = [0.0]  # host time spent inside the corr calls of the timed windows

    def window():
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step()
        host_s[0] += time.perf_counter() - t0

    windows = timed_windows(window, stream, world, min_total_ms=args.min_timed_ms)
    clk = clocks.stop()
    ms_total = statistics.median(windows)
    ms_step = ms_total / args.steps
    value = world * BATCH * args.steps / (ms_total / 1e3)
    host_ms_step = 1e3 * host_s[0] / (len(windows) * args.steps)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    # ---- per-kernel device time (separate instrumented steps) -------------
    _lib.stage_timing(True)
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    stages = _lib.stage_timing_read()
    _lib.stage_timing(False)
    kern = {}
    launches_per_step = sum(v[1] for v in stages.values()) / 2
    tot_ms = sum(v[0] for v in stages.values())
    for name, (ms, n) in stages.items():
        kern[name] = {"launches": n, "ms_per_launch": ms / max(n, 1),
                      "share": ms / tot_ms if tot_ms else None}

    # ---- end to end through the public API with host buffers --------------
    # Each step's templates are copied from pinned host memory on a side
    # stream into one of two device buffers while the previous step computes
    # (the overlap a caller streaming template batches would use); every copy
    # and every peak read-back lies inside the timed region.
    peaks_host = torch.empty((BATCH,), dtype=torch.float32).pin_memory()
    peaks = torch.empty((BATCH,), dtype=torch.float32, device=dev)
    copy_stream = torch.cuda.Stream(dev)
    tm_bufs = [tm, torch.empty_like(tm)]
    ready = [torch.cuda.Event(), torch.cuda.Event()]  # buffer i holds its step's copy
    freed = [torch.cuda.Event(), torch.cuda.Event()]  # step using buffer i has finished

    def copy_in(i):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(freed[i])
            tm_bufs[i].copy_(tm_host, non_blocking=True)
            ready[i].record(copy_stream)

    e2e_host_s = [0.0]  # host time inside the corr calls of the timed e2e run

    def e2e_run(n):
        """n steps; the first copy starts after the work already on the stream."""
        for i in (0, 1):
            freed[i].record(stream)
        copy_in(0)
        for s in range(n):
            b = s & 1
            if s + 1 < n:
                copy_in(b ^ 1)
            stream.wait_event(ready[b])
            t0 = time.perf_counter()
            zipfft.padded_rconv2d.corr(tm_bufs[b], ws, spec_T, out, H, W, peaks=peaks)
            e2e_host_s[0] += time.perf_counter() - t0
            freed[b].record(stream)
            peaks_host.copy_(peaks, non_blocking=True)

    e2e_run(args.warmup)
    torch.cuda.synchronize()
    barrier(world)
    e2e_host_s[0] = 0.0
    ev0.record(stream)
    e2e_run(args.steps)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms_rank = ev0.elapsed_time(ev1)
    e2e_ms = max_over_ranks(e2e_ms_rank, world)
    e2e_value = world * BATCH * args.steps / (e2e_ms / 1e3)

    # ---- per-rank figures for N > 1 (every rank's own device time) --------
    per_rank = None
    if world > 1:
        import torch.distributed as dist

        mine = {"rank": rank, "value": BATCH * args.steps / (ms_total / 1e3),
                "e2e": BATCH * args.steps / (e2e_ms_rank / 1e3),
                "host_ms_per_step_in_corr": host_ms_step,
                "e2e_host_ms_per_step_in_corr": 1e3 * e2e_host_s[0] / args.steps}
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        per_rank = gathered

    # ---- comparison and baselines (rank 0, N = 1) --------------------------
    cufft = cpu = spectrum = configs = None
    if rank == 0 and world == 1 and not args.skip_configs:
        del out, ws
        torch.cuda.empty_cache()
        configs = measure_configs(dev)
    if rank == 0 and world == 1 and not args.skip_baselines:
        spectrum = image_spectrum_timing(image)
        rate, ms = cufft_torch_rate(spec_nat, tm)
        cufft = {"value": rate, "unit": UNIT, "ms_per_step": ms,
                 "pipeline": "F.pad + torch.fft.rfft2 + *conj + irfft2 (cuFFT), same GPU"}
        rate, cores, n, el = cpu_reference_rate()
        cpu = {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{n} templates of this workload (4096^2 full maps) in {el:.1f} s, "
                         f"the reference test's torch.fft path (oracle) on {cores} host threads"}

    if rank == 0:
        per_gpu = value / world
        achieved = ALG_BYTES * per_gpu / 1e9
        peak, peak_src = measured_hbm_peak()
        traffic, traffic_note = measured_traffic()
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) image and soft-masked templates)",
            "config": {"workload": WORKLOAD, "image": [H, W], "template": [TH, TW],
                       "templates_per_gpu_step": BATCH, "global_batch": BATCH * world,
                       "output": "full", "parallelism": f"dp{world} (template shards)",
                       "l2": L2_NOTE, "timing": window_summary(windows)},
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": BATCH * TH * TW * 4,
                    "d2h_bytes_per_step": BATCH * 4,
                    "api": "zipfft.padded_rconv2d.corr(..., peaks=); each step's templates "
                           "copied from pinned host memory on a side stream into one of two "
                           "device buffers while the previous step computes, each template's "
                           "peak score (computed by the kernel that writes its map) read back "
                           "each step"},
            "gpu_launches": int(round(launches_per_step * args.steps)),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "traffic_source": traffic_note,
                         "unit_of_work": "one correlation (k_row_r2c + k_col_fused + k_row_c2r "
                                         "for one template)",
                         "algorithmic_bytes_per_unit": ALG_BYTES, "peak_source": peak_src},
            "kernels": kern,
            "clocks": clk,
        }
        line["host_ms_per_step_in_corr"] = host_ms_step
        if per_rank is not None:
            line["per_rank"] = per_rank
        if configs is not None:
            line["configs"] = configs
        if cufft is not None:
            line["cufft_torch"] = cufft
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if spectrum is not None:
            line["image_spectrum"] = spectrum
        print(json.dumps(line), flush=True)
    return 0


def measured_hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (of measured)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s (of fallback)"


def measured_traffic():
    """DRAM bytes (read + write) per correlation from the committed ncu
    summary, or None when that summary was captured on another build of the
    library (its `build` hash differs from the current sources')."""
    from zipfft_b200 import build as B

    path = os.path.join(ROOT, "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        value = float(d["dram_bytes_per_correlation"])
    except (OSError, KeyError, ValueError):
        return None, "no ncu traffic summary"
    cur = B.sources_hash()[:16]
    if d.get("build") != cur:
        return None, (f"stale: profiles/dram_traffic.json was captured on build "
                      f"{d.get('build')}, the library is {cur}")
    return value, f"profiles/dram_traffic.json (ncu, build {cur})"


# ---------------------------------------------------------------------------
# Search workload (--workload search): 2D template matching, max / argmax
# ---------------------------------------------------------------------------
SEARCH_TH = 384
SEARCH_BATCH = 256      # templates per corr_max call (per GPU)
SEARCH_PER_STEP = 1024  # templates per GPU per step: one search of 4 streamed batches
SEARCH_METRIC = ("2D padded cross-corr/sec folded into per-pixel max/argmax, 4096² img, "
                 "384² tmpl")
# template + spectrum per correlation; the maps are read-modified-written per
# template (max read, updated where improved)
SEARCH_ALG_BYTES = SEARCH_TH * SEARCH_TH * 4 + H * (W // 2 + 1) * 8


def search_rate(dev, steps: int, warmup: int, stats: bool = False) -> dict:
    """One GPU: template_search over SEARCH_PER_STEP templates of 384^2 (the
    search configuration's per-GPU share), streamed in batches of 256."""
    from zipfft_b200 import padded_rconv2d as P
    from zipfft_b200.search import template_search

    spec = P.image_spectrum(make_image(0).to(dev))
    g = torch.Generator().manual_seed(7)
    tm = unit_variance(torch.randn((SEARCH_PER_STEP, SEARCH_TH, SEARCH_TH), generator=g))
    tm = tm.pin_memory()

    def step():
        return template_search(tm, spec, H, W, batch_size=SEARCH_BATCH, full=True, stats=stats)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        step()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    rate = SEARCH_PER_STEP / (ms / 1e3)
    peak, peak_src = measured_hbm_peak()
    return {"workload": f"search: 4096^2 image, {SEARCH_PER_STEP} templates of {SEARCH_TH}^2 "
                        f"N(0,1) zero-mean unit-variance per GPU, streamed from pinned host "
                        f"memory in batches of {SEARCH_BATCH}, running max/argmax maps "
                        f"(one GPU's share of the 8192-template search)",
            "value": rate, "unit": UNIT, "ms_per_call": ms, "calls": steps,
            "algorithmic_bytes_per_corr": SEARCH_ALG_BYTES,
            "achieved_gbs": SEARCH_ALG_BYTES * rate / 1e9,
            "frac": SEARCH_ALG_BYTES * rate / 1e9 / peak, "peak_source": peak_src}


def run_search_arm(args, world, rank, local):
    """One step = one template_search over 1024 templates of 384^2 per GPU in
    batches of 256 (copied from pinned host memory on a side stream while
    the previous batch computes), the running max / argmax (and with --stats
    the sum and sum of squares) per pixel, and the final NCCL reduction
    across ranks."""
    from zipfft_b200 import padded_rconv2d as P
    from zipfft_b200.search import template_search

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    image = make_image(0).to(dev)
    spec = P.image_spectrum(image)
    # Each rank holds only its own shard of the template set.
    g = torch.Generator().manual_seed(7 + rank)
    tm = torch.randn((SEARCH_PER_STEP, SEARCH_TH, SEARCH_TH), generator=g)
    tm = ((tm - tm.mean(dim=(1, 2), keepdim=True)) / tm.std(dim=(1, 2), keepdim=True))
    tm = tm.contiguous().pin_memory()
    group = None
    if world > 1:
        import torch.distributed as dist

        group = dist.group.WORLD

    def step():
        return template_search(tm, spec, H, W, batch_size=SEARCH_BATCH, full=True, group=group,
                               stats=args.stats, shard_base=rank * SEARCH_PER_STEP)

    for _ in range(args.warmup):
        out = step()
    torch.cuda.synchronize()
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        out = step()
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms_total = max_over_ranks(ev0.elapsed_time(ev1), world)
    value = world * SEARCH_PER_STEP * args.steps / (ms_total / 1e3)
    # One more step, untimed, with events at the search's phase boundaries:
    # device ms per phase, max over ranks.
    marks = {}
    out = template_search(tm, spec, H, W, batch_size=SEARCH_BATCH, full=True, group=group,
                          stats=args.stats, shard_base=rank * SEARCH_PER_STEP, phase_events=marks)
    torch.cuda.synchronize()
    order = [k for k in ("start", "first_copy", "batches", "pack", "reduce", "unpack", "end")
             if k in marks]
    phases = {f"{a}->{b}": max_over_ranks(marks[a].elapsed_time(marks[b]), world)
              for a, b in zip(order, order[1:])}
    if rank == 0:
        peak, peak_src = measured_hbm_peak()
        achieved = SEARCH_ALG_BYTES * value / world / 1e9
        line = {
            "metric": SEARCH_METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) image and zero-mean unit-variance templates)",
            "config": {"workload": f"search: 4096^2 image, {SEARCH_PER_STEP} templates of "
                                   f"{SEARCH_TH}^2 per GPU per step streamed from pinned host "
                                   f"memory in batches of {SEARCH_BATCH}, running max/argmax"
                                   + (" + sum/sum of squares" if args.stats else "")
                                   + " maps (4096^2), one NCCL reduction per step",
                       "global_batch": SEARCH_PER_STEP * world,
                       "parallelism": f"dp{world} (template shards)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "algorithmic_bytes_per_unit": SEARCH_ALG_BYTES,
                         "unit_of_work": "one correlation folded into the maps",
                         "peak_source": peak_src},
            "clocks": clk,
            "phases_ms": phases,
        }
        print(json.dumps(line), flush=True)
    del out
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("zipfft", "reference"), default="zipfft")
    ap.add_argument("--skip-baselines", action="store_true",
                    help="skip the cuFFT comparison and the CPU baseline")
    ap.add_argument("--min-timed-ms", type=float, default=MIN_TIMED_MS,
                    help="repeat the timed K-step window until this much device time has "
                         "passed (default 2000 ms, so that the clock sampler sees the load); "
                         "0 times a single window (profiling captures)")
    ap.add_argument("--skip-configs", action="store_true",
                    help="skip the other measurement configurations (the `configs` object)")
    ap.add_argument("--batch", type=int, default=BATCH,
                    help="templates per GPU per step (default 32, the benchmarked workload; "
                         "smaller values only for profiling captures)")
    ap.add_argument("--workload", choices=("maps", "search"), default="maps",
                    help="maps: the full correlation maps (default, the headline); search: "
                         "the template-matching search with per-pixel max / argmax")
    ap.add_argument("--stats", action="store_true",
                    help="search workload: also accumulate per-pixel sum and sum of squares")
    args = ap.parse_args(argv)
    args.warmup = max(args.warmup, 3)  # at least 3 untimed warm-up steps; reported as run
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        return run_reference_arm(args, world, rank)
    world, rank, local = dist_setup()
    try:
        if args.workload == "search":
            return run_search_arm(args, world, rank, local)
        return run_gpu_arm(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())

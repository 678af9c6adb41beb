#!/usr/bin/env python
"""Benchmark of the B200 rasterizer hot path.  Prints one JSON line (rank 0).

Workload (BASELINE config 2 scene, config 3 views): 1.18M gaussians with the config-1 distribution,
C-channel features (default 512), SH degree 3, 979x546 views on the 64-view orbit (radius 8,
elevation 10-30 deg).  One step = every rank renders --views views (default 8) through the full
hot path -- the model's parameter activations and projection, SH colour, binning, the fused RGB +
feature blend, 0.8 L1 + 0.2 (1 - SSIM) on RGB, a fixed random gradient on the feature image (the
reference harness's scope, bench/harness.py:42-50, plus the activations of utils/gaussian.py:73-98
that its training loop runs) -- and backpropagates into every raw gaussian parameter, accumulating
over its views; with N > 1 ranks the per-gaussian gradients (59 + C floats each) are then
all-reduced over NCCL.  Scaling is weak: every rank renders its own views.  value = views / s over all ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--channels C] [--views V]
    python bench.py --impl reference ...   # the CPU oracle on a bounded sample of the same workload
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
from collections import defaultdict
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "high-dimensional-splatting_b200"))

METRIC = "fwd+bwd ms/view (1.18M gaussians, 979x546, C=32–512); views/s at 1/2/4/8 GPU"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--channels", type=int, default=512)
    ap.add_argument("--views", type=int, default=8, help="views per rank per step")
    ap.add_argument("--gaussians", type=int, default=1_180_000)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="also time fwd/bwd per C in the reference harness scope")
    return ap.parse_args()


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {**PEAKS_FALLBACK, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], 0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[4:8]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


class CallTimer:
    """Device time of every libhds_b200 entry point, bracketed by CUDA events on the launch stream."""

    def __init__(self, native):
        import torch

        self.torch = torch
        self.native = native
        self.active = False
        self.events = defaultdict(list)
        for name in list(native.SIGNATURES):
            if name.endswith("_bytes") or name in ("hds_last_error", "hds_abi_version", "hds_device_status",
                                                   "hds_launch_count"):
                continue
            fn = getattr(native.lib, name)
            setattr(native.lib, name, self._wrap(name, fn))

    def _wrap(self, name, fn):
        def call(*args):
            if not self.active:
                return fn(*args)
            stream = self.torch.cuda.current_stream()
            s = self.torch.cuda.Event(enable_timing=True)
            e = self.torch.cuda.Event(enable_timing=True)
            s.record(stream)
            rc = fn(*args)
            e.record(stream)
            self.events[name].append((s, e))
            return rc

        return call

    def totals_ms(self):
        return {name: sum(s.elapsed_time(e) for s, e in evs) for name, evs in self.events.items()}

    def counts(self):
        return {name: len(evs) for name, evs in self.events.items()}


def make_workload(args, device, rank, world):
    import torch

    from hds_b200 import parallel, scenes

    scene = scenes.config1(0, n=args.gaussians, channels=args.channels)
    cams = scenes.orbit(64)
    # Round-robin over the orbit; each rank takes args.views views per step (weak scaling).
    views = parallel.shard_views(len(cams) * args.views * world, rank, world)[:args.views]
    views = [v % len(cams) for v in views]
    gen = torch.Generator().manual_seed(100 + rank)
    h, w = cams[0].height, cams[0].width
    gt_host = [torch.randint(0, 256, (h, w, 3), dtype=torch.uint8, generator=gen).pin_memory() for _ in views]
    pose_host = [cams[v].world_to_camera.clone().pin_memory() for v in views]
    feat_grad = torch.rand(h, w, args.channels, generator=gen).to(device) / (h * w)
    # The model's raw parameters (the reference's Gaussian.params): log-scales, quaternions, opacity
    # logits; their activations run inside the projection kernels.
    op = scene.opacities.clamp(1e-6, 1 - 1e-6)
    raw = {"means": scene.means, "log_scales": torch.log(scene.scales), "quats": scene.quats,
           "opacity_logits": torch.log(op / (1 - op)), "sh_dc": scene.sh_dc, "sh_rest": scene.sh_rest,
           "features": scene.features}
    leaves = {k: v.to(device).contiguous().requires_grad_(True) for k, v in raw.items()}
    bucket = parallel.GradBucket(list(leaves.values()))
    return {"bucket": bucket, "scene": scene, "cams": cams, "views": views, "gt_host": gt_host, "pose_host": pose_host,
            "gt_dev": [g.to(device) for g in gt_host], "pose_dev": [p.to(device) for p in pose_host],
            "feat_grad": feat_grad, "leaves": leaves, "bg": torch.zeros(3, device=device)}


def render_view(wl, i, pose, gt_u8):
    """Forward + backward of one view; gradients accumulate into the leaves."""
    import torch

    from hds_b200.loss import l1_loss, ssim
    from hds_b200.projection import project_gaussians_raw
    from hds_b200.rasterizer import accumulate_leaf_grads, rasterize
    from hds_b200.sh import view_colors

    cam = wl["cams"][wl["views"][i]]
    L = wl["leaves"]
    center = -(pose[:3, :3].T @ pose[:3, 3])
    # The views of a step accumulate into the gradient bucket: the projection, SH and feature backward
    # passes add straight into it.  The projection applies the parameter activations and view_colors
    # forms normalize(means - center) inside the SH kernels.
    with accumulate_leaf_grads():
        means2D, depths, radii, conics, opacities = project_gaussians_raw(
            L["means"], L["log_scales"], L["quats"], L["opacity_logits"], pose, cam.fx, cam.fy, cam.cx, cam.cy,
            cam.width, cam.height)
        colors = view_colors(L["sh_dc"], L["sh_rest"], L["means"], center, 3, radii)
        image, feat = rasterize(means2D, depths, radii, conics, colors, opacities, cam.width, cam.height,
                                wl["bg"], L["features"])
    gt = gt_u8.float() / 255.0
    loss = 0.8 * l1_loss(image, gt) + 0.2 * (1.0 - ssim(image, gt))
    wl["bucket"].ready()  # the step's gradient clear ran on a side stream during the forward
    torch.autograd.backward([loss, feat], [None, wl["feat_grad"]])
    return loss.detach()


def run_step(wl, dist, e2e: bool):
    import torch

    losses = []
    for i in range(len(wl["views"])):
        if e2e:
            pose = wl["pose_host"][i].to(wl["feat_grad"].device, non_blocking=True)
            gt = wl["gt_host"][i].to(wl["feat_grad"].device, non_blocking=True)
        else:
            pose, gt = wl["pose_dev"][i], wl["gt_dev"][i]
        losses.append(render_view(wl, i, pose, gt))
    if dist is not None:
        wl["bucket"].all_reduce()  # one NCCL all-reduce of every per-gaussian gradient
    loss = torch.stack(losses).sum()
    if e2e:
        return loss.item()  # device -> host read of the step's result
    return loss


def zero_grads(wl):
    wl["bucket"].zero_async()


def tile_stats(wl, device):
    """Visited list length per tile (min(list length, max contributor index)) for one view, for the
    algorithmic byte / flop counts of the roofline."""
    import torch

    from hds_b200 import gaussian_rasterizer as ext
    from hds_b200.projection import project_gaussians_raw

    L = wl["leaves"]
    cam = wl["cams"][wl["views"][0]]
    with torch.no_grad():
        means2D, depths, radii, conics, opacities = project_gaussians_raw(
            L["means"], L["log_scales"], L["quats"], L["opacity_logits"], wl["pose_dev"][0], cam.fx, cam.fy, cam.cx,
            cam.cy, cam.width, cam.height)
        colors = torch.zeros_like(L["means"])
        _, _, n_contrib, values, ranges, _, _ = ext.rasterize(means2D, depths, radii, conics, colors, opacities,
                                                             wl["bg"], cam.width, cam.height)
        h, w = cam.height, cam.width
        tx, ty = (w + 15) // 16, (h + 15) // 16
        pad = torch.zeros(ty * 16, tx * 16, dtype=torch.int32, device=device)
        pad[:h, :w] = n_contrib
        tile_max = pad.reshape(ty, 16, tx, 16).amax(dim=(1, 3)).reshape(-1)
        lengths = (ranges[:, 1] - ranges[:, 0])
        visited = torch.minimum(lengths, tile_max)
    return {"pairs": int(values.numel()), "visited": int(visited.sum()), "pixels": h * w,
            "visible": int((radii > 0).sum())}


# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) from one-pass ncu captures of
# this bench's own workload: (call, channels, gaussians) -> (bytes, summary under profiles/).
MEASURED_TRAFFIC = {
    ("hds_render_backward_fused", 512, 1_180_000):  # the four-block cluster kernel (the default at C = 512)
        (2.88e9 + 0.832e9, "profiles/feature_backward_traffic_config2_1180k_c512.md"),
    ("hds_render_features_backward_accumulate", 512, 1_180_000):  # the one-block kernel
        (2.59e9 + 0.595e9, "profiles/feature_backward_traffic_config2_1180k_c512.md"),
}


def roofline(name, ms_per_launch, stats, args, peaks, n):
    """Algorithmic bytes (or flops) per launch of the dominant call over its measured duration."""
    C = args.channels
    P = stats["pixels"]
    V = stats["visited"]
    if name == "hds_render_features_forward":
        flops = 2.0 * C * 256 * V  # weights x features per visited (tile, gaussian), 256 px per tile
        tf32_peak = peaks["bf16_tflops"] / 2.0
        ach = flops / (ms_per_launch * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": ach, "peak": tf32_peak, "unit": "TFLOP/s", "frac": ach / tf32_peak,
                "traffic": None, "kernel": name,
                "peak_note": f"TF32 dense = half the {peaks['source']} cuBLAS bf16 rate"}
    if name in ("hds_render_features_backward", "hds_render_features_backward_accumulate",
                "hds_render_backward_fused"):
        nbytes = P * (4 * C + 12) + V * (4 * C + 32) + n * (4 * C + 36) * 2
        if name == "hds_render_backward_fused":  # plus the RGB terms: dL/dimage, colours and their gradient
            nbytes += P * 12 + n * 24
    elif name == "hds_render_backward":
        nbytes = P * (12 + 8) + V * 44 + n * 36 * 2
    else:
        nbytes = None
    if nbytes is None:
        return {"bound": "hbm", "achieved": None, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": None,
                "traffic": None, "kernel": name}
    ach = nbytes / (ms_per_launch * 1e-3) / 1e9
    out = {"bound": "hbm", "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": ach / peaks["hbm_gbs"],
           "traffic": None, "kernel": name, "algorithmic_bytes": nbytes}
    measured = MEASURED_TRAFFIC.get((name, C, args.gaussians))
    if measured is not None:
        out["traffic"], out["traffic_source"] = measured
    return out


CPU_WINDOW = 64  # side of the image windows the CPU oracle renders as its bounded sample
CPU_MAX_WORKERS = 64  # worker processes at most (each holds a copy of the scene geometry)
_cpu_state = None  # per worker process: the scene geometry, camera and feature table


def _cpu_worker_init(geometry, camera, channels):
    """Worker set-up, untimed: the oracle library, the scene geometry (means, scales, quats,
    opacities), the camera (pose, fx, fy, cx, cy) and a seeded [4096, C] feature table.  The
    oracle's cost does not depend on feature values, and a window is rendered with only the
    gaussians it sees (rows of the table as their features), so no [N, C] array is built per worker.
    Workers import numpy and the oracle only."""
    global _cpu_state
    import numpy as np

    sys.path.insert(0, str(REPO / "oracle"))
    import oracle

    oracle.lib()
    table = np.random.default_rng(0).random((4096, channels), dtype=np.float32)
    _cpu_state = {"oracle": oracle, "geometry": geometry, "camera": camera, "table": table, "channels": channels}


def _cpu_window(wx, wy):
    """Forward and backward of the CPU_WINDOW-square window at pixel (wx, wy) of view 0 through the
    oracle: projection of every gaussian, binning, RGB + C-channel blend, backward.  Returns seconds."""
    import numpy as np

    st = _cpu_state
    oracle, (means, scales, quats, opac) = st["oracle"], st["geometry"]
    pose, fx, fy, cx, cy = st["camera"]
    crop = CPU_WINDOW
    t0 = time.perf_counter()
    m2, dep, rad, con = oracle.project_forward(means, scales, quats, opac, pose, fx, fy, cx - wx, cy - wy, crop, crop)
    keep = np.nonzero(rad > 0)[0]
    m2, dep, rad, con, op = m2[keep], dep[keep], rad[keep], con[keep], opac[keep]
    feats = st["table"][keep % len(st["table"])]
    colors = np.full((len(keep), 3), 0.5, np.float32)
    r = oracle.rasterize(m2, dep, rad, con, colors, op, crop, crop, background=np.zeros(3), features=feats)
    g_img = np.full((crop, crop, 3), 1e-3, np.float32)
    g_feat = np.full((crop, crop, st["channels"]), 1e-3, np.float32)
    oracle.render_backward(r["ranges"], r["values"], m2, con, colors, op, crop, crop, r["final_T"], r["n_contrib"],
                           grad_image=g_img, background=np.zeros(3), features=feats, grad_features=g_feat)
    return time.perf_counter() - t0


def cpu_sample(args, rounds: int, warmup: int):
    """The CPU oracle on every usable host core: one worker process per core (started with spawn, so
    that a parent that has touched CUDA is safe), each rendering one window per round at its own
    place in the view.  Untimed warm-up rounds, then timed rounds; scaled to views/s."""
    import concurrent.futures
    import multiprocessing

    from hds_b200 import scenes

    sys.path.insert(0, str(REPO / "oracle"))
    import oracle

    oracle.lib()  # built here once, before the workers load it
    s = scenes.config1(0, n=args.gaussians, channels=0)
    geometry = tuple(t.numpy() for t in (s.means, s.scales, s.quats, s.opacities))
    cam = scenes.orbit(64)[0]
    camera = (cam.world_to_camera.numpy(), cam.fx, cam.fy, cam.cx, cam.cy)
    cols, rows = cam.width // CPU_WINDOW, cam.height // CPU_WINDOW
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    workers = min(cores, CPU_MAX_WORKERS)

    def windows(r):
        # Spread over the view's grid of windows: consecutive indices 37 windows apart.
        out = []
        for k in range(workers):
            idx = ((r * workers + k) * 37) % (cols * rows)
            out.append(((idx % cols) * CPU_WINDOW, (idx // cols) * CPU_WINDOW))
        return out

    ctx = multiprocessing.get_context("spawn")
    with concurrent.futures.ProcessPoolExecutor(max_workers=workers, mp_context=ctx, initializer=_cpu_worker_init,
                                                initargs=(geometry, camera, args.channels)) as pool:
        for r in range(warmup):
            list(pool.map(_cpu_window, *zip(*windows(r))))
        t0 = time.perf_counter()
        busy = 0.0
        for r in range(rounds):
            busy += sum(pool.map(_cpu_window, *zip(*windows(warmup + r))))
        secs = time.perf_counter() - t0
    frac = rounds * workers * CPU_WINDOW * CPU_WINDOW / (cam.width * cam.height)
    return {"value": frac / secs, "unit": "views/s", "cores": workers, "kind": "port",
            "sample": f"{rounds} rounds x {workers} processes, each a {CPU_WINDOW}x{CPU_WINDOW} window of one "
                      f"{cam.width}x{cam.height} view ({frac:.4f} views in all, windows spread over the view), "
                      f"all {s.n} gaussians projected per window, C={args.channels}, fwd+bwd, oracle/hds_oracle.c, "
                      f"{secs:.1f} s wall, {busy:.1f} s of CPU work"}, secs / max(rounds, 1)


def cpu_baseline(args):
    """The cpu_baseline object of the GPU arm's line: three timed rounds of cpu_sample."""
    return cpu_sample(args, rounds=3, warmup=1)[0]


def run_reference(args, rank, world):
    """The reference arm: the CPU oracle (the reference's path restated in C; its own CPU code is Python
    that cannot travel) on all host cores, W untimed and K timed rounds of cpu_sample."""
    if rank != 0:
        return
    base, secs_per_round = cpu_sample(args, rounds=max(args.steps, 1), warmup=max(args.warmup, 0))
    line = {"metric": METRIC, "value": base["value"], "unit": "views/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * secs_per_round, "ms_per_view": 1000.0 / base["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "config2 scene, orbit views, bounded CPU sample", "channels": args.channels,
                       "gaussians": args.gaussians},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "views/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as tdist

        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        dist = tdist
    from hds_b200 import native

    timer = CallTimer(native)
    wl = make_workload(args, device, rank, world)
    n = args.gaussians

    for _ in range(args.warmup):
        zero_grads(wl)
        run_step(wl, dist, e2e=False)
    torch.cuda.synchronize()

    def timed(e2e: bool, record_calls: bool):
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        timer.active = record_calls
        launches0 = native.lib.hds_launch_count()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            zero_grads(wl)
            run_step(wl, dist, e2e=e2e)
        end.record()
        torch.cuda.synchronize()
        timer.active = False
        timed.launches = native.lib.hds_launch_count() - launches0
        ms = start.elapsed_time(end)
        if dist is not None:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        return ms

    clocks = ClockSampler(local)
    clocks.start()
    ms = timed(e2e=False, record_calls=True)
    launches = timed.launches
    clock_info = clocks.stop()
    calls = timer.totals_ms()
    counts = timer.counts()
    total_views = args.steps * args.views * world
    value = total_views / (ms / 1000.0)
    e2e = None
    if not args.no_e2e:
        ms_e2e = timed(e2e=True, record_calls=False)
        h2d = sum(g.numel() for g in wl["gt_host"]) + sum(p.numel() * 4 for p in wl["pose_host"])
        e2e = {"value": total_views / (ms_e2e / 1000.0), "unit": "views/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": 4}

    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return

    peaks = load_peaks()
    stats = tile_stats(wl, device)
    kernel_calls = {k: v for k, v in calls.items()}
    dominant = max(kernel_calls, key=kernel_calls.get)
    per_launch = kernel_calls[dominant] / max(1, counts[dominant])
    roof = roofline(dominant, per_launch, stats, args, peaks, n)
    line = {
        "metric": METRIC, "value": value, "unit": "views/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "ms_per_view": ms / (args.steps * args.views),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (feature blend tf32)",
        "data": "synthetic (seeded config-1 distribution; the Truck scene is not available)",
        "config": {"workload": "config2 scene (1.18M gaussians), config3 orbit views, 979x546, full fwd+bwd step",
                   "gaussians": n, "channels": args.channels, "views_per_gpu_per_step": args.views,
                   "sh_degree": 3, "parallelism": f"dp{world}", "l2": "inputs larger than L2 (features "
                   f"{n * args.channels * 4 / 1e9:.2f} GB)"},
        "roofline": roof,
        "call_ms_per_step": {k: v / args.steps for k, v in sorted(calls.items(), key=lambda kv: -kv[1])},
        "gpu_launches": launches,
        "tile_stats": stats,
        "clocks": clock_info,
        "e2e": e2e,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args)
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

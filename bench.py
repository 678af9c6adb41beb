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

On one GPU the line also carries the config-2 channel sweep (C = 32 ... 512, forward and backward
timed separately in the reference harness's scope, median of 50 after 10 warm-ups) and the CPU
oracle's rate on the host cores (cpu_baseline).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--channels C] [--views V] [--no-sweep]
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
    ap.add_argument("--no-sweep", action="store_true",
                    help="skip the channel sweep (fwd and bwd per C in the reference harness scope; 1 GPU only)")
    ap.add_argument("--split", choices=["views", "rows"], default="views",
                    help="views: data parallel over views (config 2/3, default); rows: one config-4 view split by "
                         "tile rows across the ranks (4M gaussians, 1920x1080, C=512 unless overridden)")
    ap.add_argument("--row-owners", choices=["bands", "blocks"], default="bands",
                    help="--split rows: which feature rows each rank owns -- bands: the scene is ordered once by the "
                         "band holding each gaussian's projected centre (band_split.band_order), so a band fetches "
                         "only the rows of gaussians that reach across its edges; blocks: equal blocks of the "
                         "scene's own order")
    ap.add_argument("--band-weights", choices=["pairs", "visited", "cost"], default="visited",
                    help="--split rows: tile-row weights the bands are balanced by -- pairs: (tile, gaussian) pairs; "
                         "visited: the list entries the blend and backward walk (per half tile, up to its last "
                         "contributor); cost: 0.69 the row's share of the visited entries + 0.31 its share of the "
                         "projected centres (the feature rows its band owns and steps under --row-owners bands), the "
                         "split of a one-GPU step between blend + backward (22.1 ms) and the feature Adam (9.9 ms)")
    args = ap.parse_args()
    if args.split == "rows" and "--gaussians" not in sys.argv:
        args.gaussians = 4_000_000
    return args


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

    from hds_b200 import optim, parallel, scenes

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
    # The step ends with the training loop's optimizer step (main.py:194): one fused Adam kernel over
    # every parameter, at the reference's learning rates (the means' scaled by a scene extent of 5).
    # With N ranks the gradients are reduce-scattered, each rank steps its 1/N of the parameters and
    # the stepped shards are all-gathered (ShardedFlatAdam): an all-reduce's traffic, 1/N of the
    # optimizer's memory traffic per rank.
    lrs = [optim.REFERENCE_LRS[k] * (5.0 if k == "means" else 1.0) for k in leaves]
    if world > 1:
        opt = optim.ShardedFlatAdam(list(leaves.values()), lrs, eps=1e-15)
    else:
        opt = optim.FlatAdam(list(leaves.values()), lrs, eps=1e-15)
    bucket = opt.bucket
    return {"bucket": bucket, "optimizer": opt, "scene": scene, "cams": cams, "views": views, "gt_host": gt_host, "pose_host": pose_host,
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
    wl["optimizer"].step()  # with N ranks: reduce-scatter, Adam on this rank's shard, all-gather
    loss = torch.stack(losses).sum()
    if e2e:
        return loss.item()  # device -> host read of the step's result
    return loss


def zero_grads(wl):
    wl["bucket"].zero_async()


def tile_stats(wl, device):
    """Counts of one view of the step, for the algorithmic byte / flop models of the rooflines."""
    import torch

    from hds_b200.projection import project_gaussians_raw

    L = wl["leaves"]
    cam = wl["cams"][wl["views"][0]]
    with torch.no_grad():
        means2D, depths, radii, conics, opacities = project_gaussians_raw(
            L["means"], L["log_scales"], L["quats"], L["opacity_logits"], wl["pose_dev"][0], cam.fx, cam.fy, cam.cx,
            cam.cy, cam.width, cam.height)
    return projected_stats(means2D, depths, radii, conics, opacities, cam, device)


def projected_stats(means2D, depths, radii, conics, opacities, cam, device):
    """Pixels P, duplicated (tile, gaussian) pairs D, visited pairs V (per tile, min(list length, the
    tile's largest contributor count)) and visible gaussians of one projected view."""
    import torch

    from hds_b200 import gaussian_rasterizer as ext

    with torch.no_grad():
        colors = torch.zeros_like(conics)
        bg = torch.zeros(3, device=device)
        _, _, n_contrib, values, ranges, _, _ = ext.rasterize(means2D, depths, radii, conics, colors, opacities,
                                                             bg, cam.width, cam.height)
        h, w = cam.height, cam.width
        tx, ty = (w + 15) // 16, (h + 15) // 16
        pad = torch.zeros(ty * 16, tx * 16, dtype=torch.int32, device=device)
        pad[:h, :w] = n_contrib
        tile_max = pad.reshape(ty, 16, tx, 16).amax(dim=(1, 3)).reshape(-1)
        lengths = (ranges[:, 1] - ranges[:, 0])
        visited = torch.minimum(lengths, tile_max)
    return {"pairs": int(values.numel()), "visited": int(visited.sum()), "pixels": h * w,
            "visible": int((radii > 0).sum())}


# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum), from one-pass ncu captures of
# two small cases of this bench's workload (one view, C = 512, 100K and 300K gaussians), fitted as
# a + b V in the visited (tile, gaussian) pairs V and evaluated at the run's V: the per-pixel terms
# (dL/dout, the image) are the constant, the feature rows read and reduced per visited pair the slope.
# The backward's figure is the cluster kernel plus its one-block helper.  (call, channels) ->
# (a bytes, b bytes per visited pair, summary under profiles/).
TRAFFIC_FIT = {
    ("hds_render_backward_fused", 512): (0.978e9, 2585.0, "profiles/feature_backward_traffic_fit_c512.md"),
    ("hds_render_features_forward", 512): (0.966e9, 907.0, "profiles/feature_backward_traffic_fit_c512.md"),
}

# The algorithmic model of each stage of one view (the hot-path table's measurement row): bytes that
# must cross HBM, or tensor flops for the feature blend.  P pixels, V visited (tile, gaussian) pairs
# (min(list length, the tile's last contributor)), D duplicated (tile, gaussian) pairs, n gaussians,
# vis visible gaussians, C channels.
STAGES = {
    "preprocess": ("hds_project_forward_raw", "hds_eval_sh_forward_view"),
    "binning": ("hds_rasterize_prepare", "hds_rasterize_sort"),
    "feature_forward": ("hds_render_features_forward",),
    "backward": ("hds_render_backward_fused", "hds_render_features_backward", "hds_render_features_backward_accumulate",
                 "hds_render_backward"),
    "preprocess_backward": ("hds_project_backward_raw", "hds_eval_sh_backward_view"),
    "ssim_forward": ("hds_ssim_forward",),
    "ssim_backward": ("hds_ssim_backward",),
    "optimizer": ("hds_adam_step",),  # once per step, not per view
}


def stage_model(stage, st, C, n, rgb_terms=True, world=1):
    """(bound, algorithmic bytes or flops, formula) of one view's stage."""
    P, V, D, vis = st["pixels"], st["visited"], st["pairs"], st["visible"]
    if stage == "preprocess":
        return "hbm", 84 * n + 192 * vis, "84 B/gaussian + 192 B of SH per visible gaussian"
    if stage == "binning":
        return "hbm", 48 * n + 44 * D, "48 B/gaussian + 44 B per duplicated pair"
    if stage == "feature_forward":
        return "tensor", 2.0 * C * 256 * V, "2 C 256 V flops (weights x features per visited tile-gaussian pair)"
    if stage == "backward":
        b = P * (4 * C + 12) + V * (4 * C + 32) + n * (4 * C + 36) * 2
        if rgb_terms:
            b += P * 12 + n * 24
        return "hbm", b, "P(4C+12) + V(4C+32) + 2n(4C+36) (+ 12P + 24n for the RGB terms)"
    if stage == "preprocess_backward":
        return "hbm", 172 * n + 624 * vis, ("projection backward 156 B/gaussian (accumulating), SH backward 16 "
                                            "B/gaussian + 624 B per visible gaussian (SH read, gradient added)")
    if stage in ("ssim_forward", "ssim_backward"):
        return "hbm", 72 * P, "72 B per pixel (3 channels x 4 B x 6 maps)"
    if stage == "optimizer":
        if world > 1:  # ShardedFlatAdam: each rank steps 1/world of the parameters
            return "hbm", 28 * (59 + C) * n / world, (f"28 B per parameter of this rank's 1/{world} shard (param, "
                                                      "2 moments, grad in; param, 2 moments out)")
        return "hbm", 28 * (59 + C) * n, "28 B per parameter (param, 2 moments, grad in; param, 2 moments out)"
    raise KeyError(stage)


def rooflines(call_ms, counts, launches_per_view, st, C, n, peaks, world=1):
    """Per stage of one view (the optimizer: of one step): device time (CUDA events on the launch
    stream, per launch of each of the stage's calls, summed), algorithmic bytes or flops, and the
    fraction of the measured peak."""
    out = {}
    for stage, calls in STAGES.items():
        ms = sum(call_ms.get(c, 0.0) / max(1, counts.get(c, 0)) * launches_per_view.get(c, 0) for c in calls)
        if ms <= 0:
            continue
        bound, amount, formula = stage_model(stage, st, C, n, world=world)
        if bound == "tensor":
            peak = peaks["bf16_tflops"] / 2.0
            ach = amount / (ms * 1e-3) / 1e12
            out[stage] = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                          "ms": ms, "flops": amount, "model": formula,
                          "peak_note": f"TF32 dense = half the {peaks['source']} cuBLAS bf16 burst rate"}
        else:
            ach = amount / (ms * 1e-3) / 1e9
            out[stage] = {"bound": "hbm", "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                          "frac": ach / peaks["hbm_gbs"], "ms": ms, "bytes": amount, "model": formula,
                          "peak_note": f"{peaks['source']} HBM copy rate"}
    return out


CPU_WINDOW = 64  # side of the image windows the CPU oracle blends as its bounded sample
CPU_WINDOWS = 16  # fixed windows of view 0, spread over the image (the same every round and in both legs)
CPU_MAX_WORKERS = 64  # worker processes at most (each holds a copy of the scene geometry)
CPU_ADAM_SAMPLE = 1 << 22  # elements of the per-worker Adam sample
_cpu_state = None  # per worker process: scene slice, full-view projection, window subsets, feature table


def _cpu_windows(width, height):
    """CPU_WINDOWS window origins on the view's grid of whole 64 x 64 windows, stratified: every k-th
    window in row-major order, so that dense and sparse parts of the view are both sampled.  Origins
    are multiples of 64, so a window's tiles are tiles of the full image."""
    cols, rows = width // CPU_WINDOW, height // CPU_WINDOW
    total = cols * rows
    picks = [(i * total) // CPU_WINDOWS + (total // CPU_WINDOWS) // 2 for i in range(CPU_WINDOWS)]
    return [((k % cols) * CPU_WINDOW, (k // cols) * CPU_WINDOW) for k in picks]


def _cpu_worker_init(raw, sh, camera, channels, workers, rank):
    """Worker set-up, untimed: the oracle library, the raw parameters of every gaussian (means,
    log-scales, quaternions, opacity logits) and the SH of this worker's slice, the camera, one
    full-view projection (the windows blend from it), each window's candidate gaussians, and a
    seeded [4096, C] feature table (the oracle's cost does not depend on feature values, so rows of
    the table stand in for each gaussian's features; no [N, C] array per worker).  Workers import
    numpy and the oracle only."""
    global _cpu_state
    import numpy as np

    sys.path.insert(0, str(REPO / "oracle"))
    import oracle

    oracle.lib()
    means, log_scales, quats, logits = raw
    pose, fx, fy, cx, cy, width, height = camera
    n = means.shape[0]
    lo, hi = (n * rank) // workers, (n * (rank + 1)) // workers
    scales, unit, opac = oracle.activate(log_scales, quats, logits)
    m2, dep, rad, con = oracle.project_forward(means, scales, unit, opac, pose, fx, fy, cx, cy, width, height)
    # Candidates of a window: visible gaussians whose 3.4-sigma box (beyond the opacity-aware box,
    # whose factor is at most sqrt(2 ln 255) < 3.34 sigma) meets the window; the window's own
    # binning then applies the exact test.
    reach = rad * np.float32(3.4 / 3.0) + np.float32(1.0)
    subsets = {}
    for wx, wy in _cpu_windows(width, height):
        keep = (rad > 0) & (m2[:, 0] + reach >= wx) & (m2[:, 0] - reach <= wx + CPU_WINDOW) \
            & (m2[:, 1] + reach >= wy) & (m2[:, 1] - reach <= wy + CPU_WINDOW)
        subsets[(wx, wy)] = np.nonzero(keep)[0]
    table = np.random.default_rng(0).random((4096, channels), dtype=np.float32)
    gt = np.random.default_rng(1).random((CPU_WINDOW, CPU_WINDOW, 3), dtype=np.float32)
    adam = [np.random.default_rng(2).standard_normal(CPU_ADAM_SAMPLE).astype(np.float32) for _ in range(4)]
    _cpu_state = {"oracle": oracle, "slice": (lo, hi), "raw": raw, "sh": sh, "camera": camera, "adam": adam,
                  "proj": (m2, dep, rad, con, opac), "subsets": subsets, "table": table, "gt": gt,
                  "channels": channels}


def _cpu_slice(_):
    """Per-gaussian work of one view for this worker's slice, forward and backward: activations,
    projection, view directions and SH colour, the slice's binning against the full view, then the
    SH, view-direction, projection and activation backward passes.  Returns seconds."""
    import numpy as np

    st = _cpu_state
    oracle = st["oracle"]
    lo, hi = st["slice"]
    means, log_scales, quats, logits = (a[lo:hi] for a in st["raw"])
    sh_dc, sh_rest = st["sh"]
    pose, fx, fy, cx, cy, width, height = st["camera"]
    center = -(pose[:3, :3].T @ pose[:3, 3])
    t0 = time.perf_counter()
    scales, unit, opac = oracle.activate(log_scales, quats, logits)
    m2, dep, rad, con = oracle.project_forward(means, scales, unit, opac, pose, fx, fy, cx, cy, width, height)
    dirs, s = oracle.view_dirs(means, center)
    oracle.eval_sh(sh_dc, sh_rest, dirs, 3, rad)
    oracle.bin_gaussians(m2, dep, rad, con, opac, width, height)
    k = hi - lo
    g2, gc = np.full((k, 2), 1e-3, np.float32), np.full((k, 3), 1e-3, np.float32)
    _, _, gdirs = oracle.eval_sh_backward(np.full((k, 3), 1e-3, np.float32), sh_dc, sh_rest, dirs, 3, rad)
    oracle.view_dirs_backward(gdirs, dirs, s)
    _, gs, gq = oracle.project_backward(g2, gc, means, scales, unit, pose, fx, fy, cx, cy, width, height)
    oracle.activate_backward(log_scales, quats, logits, gs, gq, np.full(opac.shape, 1e-3, np.float32))
    return time.perf_counter() - t0


def _cpu_adam(_):
    """The optimizer step's share of this worker's slice: one oracle Adam step over a fixed
    CPU_ADAM_SAMPLE-element buffer, scaled to the slice's (59 + C) parameters per gaussian.  Returns
    seconds."""
    st = _cpu_state
    p, m, v, g = st["adam"]
    lo, hi = st["slice"]
    t0 = time.perf_counter()
    st["oracle"].adam(p, m, v, g, 1, 1e-3, 0.9, 0.999, 1e-15)
    return (time.perf_counter() - t0) * (hi - lo) * (59 + st["channels"]) / CPU_ADAM_SAMPLE


def _cpu_window(wx, wy):
    """Per-pixel work of one CPU_WINDOW-square window of view 0, forward and backward: binning of
    the window's candidates, the RGB + C-channel blend, SSIM forward and backward of the window,
    and the blend's backward.  Returns seconds."""
    import numpy as np

    st = _cpu_state
    oracle = st["oracle"]
    m2, dep, rad, con, opac = st["proj"]
    keep = st["subsets"][(wx, wy)]
    crop = CPU_WINDOW
    t0 = time.perf_counter()
    m2w = m2[keep] - np.array([wx, wy], np.float32)
    dep_w, rad_w, con_w, op_w = dep[keep], rad[keep], con[keep], opac[keep]
    feats = st["table"][keep % len(st["table"])]
    colors = np.full((len(keep), 3), 0.5, np.float32)
    r = oracle.rasterize(m2w, dep_w, rad_w, con_w, colors, op_w, crop, crop, background=np.zeros(3), features=feats)
    ssim = oracle.ssim_forward(r["image"], st["gt"])
    g_img = oracle.ssim_backward(np.float32(-0.2 / (crop * crop * 3)), r["image"], st["gt"], *ssim[1:])
    g_feat = np.full((crop, crop, st["channels"]), 1e-3, np.float32)
    oracle.render_backward(r["ranges"], r["values"], m2w, con_w, colors, op_w, crop, crop, r["final_T"],
                           r["n_contrib"], grad_image=g_img, background=np.zeros(3), features=feats,
                           grad_features=g_feat)
    return time.perf_counter() - t0


def cpu_sample(args, rounds: int, warmup: int):
    """The CPU oracle on every usable host core, one worker process per core (started with spawn, so
    that a parent that has touched CUDA is safe).  A round restates one view of the bench's step on
    the CPU, split in two timed phases:
      A. per-gaussian work: every worker runs its 1/workers slice of all gaussians (activations,
         projection, SH, binning, and their backward passes) -- a whole view's worth;
      B. per-pixel work: the CPU_WINDOWS fixed 64 x 64 windows of the view (a fraction f of its
         pixels) are blended forward and backward with SSIM, one task per window.
    plus the optimizer step (one Adam pass over all parameters per step of args.views views, timed
    on a fixed sample per worker and scaled to its slice).  A view then costs
    T_A + T_adam / views + T_B / f seconds of wall time on these cores.  Untimed warm-up rounds, then
    timed rounds, all on the same windows."""
    import concurrent.futures
    import multiprocessing

    import torch

    from hds_b200 import scenes

    sys.path.insert(0, str(REPO / "oracle"))
    import oracle

    oracle.lib()  # built here once, before the workers load it
    s = scenes.config1(0, n=args.gaussians, channels=0)
    op = s.opacities.clamp(1e-6, 1 - 1e-6)
    raw = tuple(t.numpy() for t in (s.means, torch.log(s.scales), s.quats, torch.log(op / (1 - op))))
    cam = scenes.orbit(64)[0]
    camera = (cam.world_to_camera.numpy(), cam.fx, cam.fy, cam.cx, cam.cy, cam.width, cam.height)
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    workers = min(cores, CPU_MAX_WORKERS)
    windows = _cpu_windows(cam.width, cam.height)
    f = len(windows) * CPU_WINDOW * CPU_WINDOW / (cam.width * cam.height)
    ctx = multiprocessing.get_context("spawn")
    pools = []
    try:
        # One pool per slice so that worker k always owns slice k; the window tasks go to all of them.
        for rank in range(workers):
            lo, hi = (s.n * rank) // workers, (s.n * (rank + 1)) // workers
            sh = (s.sh_dc[lo:hi].numpy(), s.sh_rest[lo:hi].numpy())
            pools.append(concurrent.futures.ProcessPoolExecutor(
                max_workers=1, mp_context=ctx, initializer=_cpu_worker_init,
                initargs=(raw, sh, camera, args.channels, workers, rank)))

        def run_round():
            t0 = time.perf_counter()
            busy_a = sum(fut.result() for fut in [p.submit(_cpu_slice, 0) for p in pools])
            t_a = time.perf_counter() - t0
            # The slowest worker's scaled Adam time stands for the parallel optimizer step.
            adam = [fut.result() for fut in [p.submit(_cpu_adam, 0) for p in pools]]
            t0 = time.perf_counter()
            futs = [pools[i % workers].submit(_cpu_window, wx, wy) for i, (wx, wy) in enumerate(windows)]
            busy_b = sum(fut.result() for fut in futs)
            return t_a, max(adam), time.perf_counter() - t0, busy_a + sum(adam) + busy_b

        # Start every worker (its set-up runs in the initializer) before anything is timed.
        for fut in [p.submit(time.perf_counter) for p in pools]:
            fut.result()
        for _ in range(warmup):
            run_round()
        t_a = t_o = t_b = busy = 0.0
        for _ in range(rounds):
            a, o, b, c = run_round()
            t_a, t_o, t_b, busy = t_a + a, t_o + o, t_b + b, busy + c
    finally:
        for p in pools:
            p.shutdown()
    # The optimizer steps once per step of args.views views.
    secs_per_view = (t_a + t_o / args.views + t_b / f) / max(rounds, 1)
    return {"value": 1.0 / secs_per_view, "unit": "views/s", "cores": workers, "kind": "port",
            "sample": f"{rounds} timed rounds after {warmup} untimed, {workers} processes; a round = one view's "
                      f"per-gaussian work on all {s.n} gaussians (activations, projection, SH, binning, backward; "
                      f"{t_a / max(rounds, 1):.3f} s wall) + one Adam step over all (59 + C) parameters per gaussian "
                      f"per {args.views} views ({t_o / max(rounds, 1):.3f} s wall per step, from a "
                      f"{CPU_ADAM_SAMPLE}-element sample per worker) + the blend fwd+bwd with SSIM of {len(windows)} fixed "
                      f"{CPU_WINDOW}x{CPU_WINDOW} windows = {f:.4f} of the {cam.width}x{cam.height} view "
                      f"({t_b / max(rounds, 1):.3f} s wall, scaled by 1/{f:.4f}); C={args.channels}, "
                      f"oracle/hds_oracle.c, {busy:.1f} s of CPU work in all"}, secs_per_view


def cpu_baseline(args):
    """The cpu_baseline object of the GPU arm's line: cpu_sample with the run's own rounds, as the
    reference arm uses."""
    return cpu_sample(args, rounds=max(args.steps, 1), warmup=max(args.warmup, 0))[0]


def run_reference(args, rank, world):
    """The reference arm: the CPU oracle (the reference's path restated in C; its own CPU code is Python
    that cannot travel) on all host cores, W untimed and K timed rounds of cpu_sample.  Under torchrun
    only rank 0 runs; it reports one view per round at the GPU arm's config."""
    if rank != 0:
        return
    base, secs_per_view = cpu_sample(args, rounds=max(args.steps, 1), warmup=max(args.warmup, 0))
    line = {"metric": METRIC, "value": base["value"], "unit": "views/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * secs_per_view * args.views,
            "ms_per_view": 1000.0 * secs_per_view,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": DATA, "impl": "reference", "config": bench_config(args, args.gpus),
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "views/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


SWEEP_CHANNELS = (32, 64, 128, 256, 512)
DATA = "synthetic (seeded config-1 distribution; the Truck scene is not available)"


def bench_config(args, world):
    """The config object both arms print (the GPU arm and --impl reference)."""
    return {"workload": "config2 scene (1.18M gaussians), config3 orbit views, 979x546, full fwd+bwd step",
            "gaussians": args.gaussians, "channels": args.channels, "views_per_gpu_per_step": args.views,
            "sh_degree": 3, "parallelism": f"dp{world}",
            "l2": f"inputs larger than L2 (features {args.gaussians * args.channels * 4 / 1e9:.2f} GB)"}


def harness_time_ms(fn, before=None, iters=50, warmup=10):
    """Median device time of fn over `iters` runs after `warmup`, each bracketed by CUDA events, with a
    pause of 1.5x the last run between runs (bench/harness.py:133-154 of the reference)."""
    import torch

    for _ in range(warmup):
        if before:
            before()
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if before:
            before()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
        time.sleep(max(0.002, 1.5 * times[-1] / 1000))
    return statistics.median(times)


def harness_sweep(args, device, timer, peaks):
    """The config-2 channel sweep in the reference benchmark's scope (bench/harness.py:59-66, 133-177):
    projection (quaternions normalised by torch, as the harness does) and rasterize with features,
    colours as a leaf, forward and backward timed separately, each the median of 50 runs after 10
    warm-ups.  1.18M gaussians of the config-1 distribution, its 979x546 view, features N(0, 1),
    uniform random gradients of both images.  Per channel count it also reports the feature blend's
    and the backward's device time per call (CUDA events around each entry point) against their
    rooflines."""
    import torch
    import torch.nn.functional as F

    from hds_b200 import scenes
    from hds_b200.projection import project_gaussians
    from hds_b200.rasterizer import rasterize

    s = scenes.config1(0, n=args.gaussians, channels=0)
    cam = s.cameras[0].to(device)
    g = torch.Generator().manual_seed(0)
    base = {"means": s.means, "scales": s.scales, "quats": s.quats, "opacities": s.opacities[:, 0].contiguous(),
            "colors": torch.rand(s.n, 3, generator=g)}
    base = {k: v.to(device) for k, v in base.items()}
    grad_image = torch.rand(cam.height, cam.width, 3, generator=g).to(device)
    stats = None
    rows = {}
    for C in SWEEP_CHANNELS:
        leaves = {k: v.clone().requires_grad_(True) for k, v in base.items()}
        leaves["features"] = torch.randn(s.n, C, generator=g).to(device).requires_grad_(True)
        grad_feat = torch.rand(cam.height, cam.width, C, generator=g).to(device)
        state = {}

        def forward():
            m2, d, r, c = project_gaussians(leaves["means"], leaves["scales"], F.normalize(leaves["quats"], dim=-1),
                                            leaves["opacities"][:, None], cam.world_to_camera, cam.fx, cam.fy, cam.cx,
                                            cam.cy, cam.width, cam.height)
            state["out"] = rasterize(m2, d, r, c, leaves["colors"], leaves["opacities"][:, None], cam.width,
                                     cam.height, features=leaves["features"])

        def backward():
            torch.autograd.backward(state["out"], [grad_image, grad_feat])

        def reset():
            for leaf in leaves.values():
                leaf.grad = None
            forward()

        timer.events.clear()
        timer.active = True
        fwd = harness_time_ms(forward)
        timer.active = False
        f_calls, f_counts = timer.totals_ms(), timer.counts()
        timer.events.clear()
        timer.active = True
        bwd = harness_time_ms(backward, before=reset)
        timer.active = False
        b_calls, b_counts = timer.totals_ms(), timer.counts()
        timer.events.clear()
        if stats is None:
            with torch.no_grad():
                m2, d, r, c = project_gaussians(base["means"], base["scales"], F.normalize(base["quats"], dim=-1),
                                                base["opacities"][:, None], cam.world_to_camera, cam.fx, cam.fy,
                                                cam.cx, cam.cy, cam.width, cam.height)
            stats = projected_stats(m2, d, r, c, base["opacities"][:, None], cam, device)
        # The backward timing's calls include the untimed forwards of reset(); keep its backward calls.
        calls = {k: v for k, v in f_calls.items()}
        counts = {k: v for k, v in f_counts.items()}
        for k in STAGES["backward"] + STAGES["preprocess_backward"]:
            if k in b_calls:
                calls[k], counts[k] = b_calls[k], b_counts[k]
        per_view = {k: 1 for k in calls}
        roof = rooflines(calls, counts, per_view, stats, C, s.n, peaks)
        rows[str(C)] = {"fwd_ms": fwd, "bwd_ms": bwd, "fwd_bwd_ms": fwd + bwd,
                        "feature_forward": {k: roof["feature_forward"][k] for k in ("ms", "achieved", "unit", "frac")}
                        if "feature_forward" in roof else None,
                        "backward": {k: roof["backward"][k] for k in ("ms", "achieved", "unit", "frac")}
                        if "backward" in roof else None}
        del leaves, grad_feat, state
        torch.cuda.empty_cache()
    return {"scope": "projection + rasterize with features, colours as a leaf (bench/harness.py:59-66); median of "
                     "50 after 10 warm-ups, fwd and bwd separately (harness.py:133-177)",
            "scene": f"config2: {s.n} gaussians, one {cam.width}x{cam.height} view, features N(0,1)",
            "tile_stats": stats, "channels": rows}


def feature_block_init(device, channels, block=1 << 16, seed=1000):
    """Feature rows [start, end) of a table drawn N(0, 1) in fixed blocks of rows, each from its own
    seeded device generator: the table does not depend on how it is split over ranks."""
    import torch

    def init(start, end):
        out = torch.empty(end - start, channels, device=device)
        for b in range(start // block, (end + block - 1) // block):
            g = torch.Generator(device=device).manual_seed(seed + b)
            rows = torch.randn(block, channels, generator=g, device=device)
            lo, hi = max(start, b * block), min(end, (b + 1) * block)
            out[lo - start:hi - start] = rows[lo - b * block:hi - b * block]
        return out

    return init


def feature_rows_init(device, channels, perm, block=1 << 16, seed=1000):
    """feature_block_init for a scene whose rows were permuted: row i of the table is the seeded row of
    global id perm[i]."""
    import torch

    def init(start, end):
        ids = perm[start:end].to(device)
        out = torch.empty(ids.numel(), channels, device=device)
        blk = ids // block
        for b in torch.unique(blk).tolist():
            g = torch.Generator(device=device).manual_seed(seed + b)
            rows = torch.randn(block, channels, generator=g, device=device)
            sel = torch.nonzero(blk == b).squeeze(1)
            out[sel] = rows[ids[sel] - b * block]
        return out

    return init


def run_band_split(args, device, rank, world, dist, timer):
    """--split rows: BASELINE config 4, one view split by tile rows (hds_b200.band_split).  4M gaussians
    (80% in 200 dense clusters), one 1920x1080 view, C-channel features; every step renders the view
    once over all ranks (strong scaling) -- projection, SH, band binning and blend, 0.8 L1 + 0.2 (1 -
    SSIM) with the SSIM halo exchange, a fixed feature-image gradient, the backward, the feature
    gradients combined at their owners, the sharded geometry/SH Adam step (reduce-scatter, Adam,
    all-gather) and the feature Adam step.  Bands are balanced by the list entries the blend and
    backward walk per tile row, from a first render (--band-weights); the feature table is split in
    contiguous row blocks, rendered in place (band_split.bin_band_in_place).  With --row-owners bands
    (the default) the scene is first ordered by band (band_split.band_order), so that each rank's
    block holds its band's gaussians and only rows reaching across a band edge are fetched."""
    import torch

    from hds_b200 import band_split, gaussian_rasterizer, optim, scenes
    from hds_b200.projection import project_gaussians_raw

    s = scenes.config4(0, channels=0, n=args.gaussians)
    cam = s.cameras[0].to(device)
    H, W, C = cam.height, cam.width, args.channels
    op = s.opacities.clamp(1e-6, 1 - 1e-6)
    raw = {"means": s.means, "log_scales": torch.log(s.scales), "quats": s.quats,
           "opacity_logits": torch.log(op / (1 - op)), "sh_dc": s.sh_dc, "sh_rest": s.sh_rest}
    raw = {k: v.to(device).contiguous().requires_grad_(True) for k, v in raw.items()}
    with torch.no_grad():
        m2, dep, rad, con, opa = project_gaussians_raw(raw["means"], raw["log_scales"], raw["quats"],
                                                       raw["opacity_logits"], cam.world_to_camera, cam.fx, cam.fy,
                                                       cam.cx, cam.cy, W, H)
        _, _, ranges = gaussian_rasterizer.bin_gaussians(m2, dep, rad, con, opa, W, H)
        tx = (W + 15) // 16
        per_row = (ranges[:, 1] - ranges[:, 0]).reshape(-1, tx).sum(dim=1).double()
        weights = (per_row + 1.0).tolist()
        ty = per_row.numel()
        if args.band_weights in ("visited", "cost"):
            colors = torch.zeros(s.n, 3, device=device)
            n_contrib = gaussian_rasterizer.rasterize(m2, dep, rad, con, colors, opa, torch.zeros(3, device=device),
                                                      W, H)[2]
            padded = torch.zeros(ty * 16, tx * 16, dtype=torch.int32, device=device)
            padded[:H, :W] = n_contrib
            walked = padded.view(ty * 2, 8, tx, 16).amax(dim=(1, 3))  # per half tile: entries walked
            visited = walked.view(ty, 2 * tx).sum(dim=1).double()
            weights = (visited + 1.0).tolist()
        if args.band_weights == "cost":
            vis = rad > 0
            rows_of = (m2[vis, 1].clamp(0.0, H - 1.0) // 16).long()
            centres = torch.bincount(rows_of, minlength=ty).double()
            share = 0.69 * visited / visited.sum().clamp(min=1.0) + 0.31 * centres / centres.sum().clamp(min=1.0)
            weights = (share + 1e-9).tolist()
        starts, init = None, feature_block_init(device, C)
        if world > 1 and args.row_owners == "bands":
            from hds_b200.parallel import row_bands

            perm, starts = band_split.band_order(m2, rad, row_bands(H, world, weights))
            # The same scene in band order: every parameter row moves with its gaussian.
            raw = {k: v.detach()[perm].contiguous().requires_grad_(True) for k, v in raw.items()}
            init = feature_rows_init(device, C, perm)
    features = band_split.FeatureShards(s.n, C, rank, world, device, init=init, starts=starts)
    lrs = [optim.REFERENCE_LRS[k] * (5.0 if k == "means" else 1.0) for k in raw] + [optim.REFERENCE_LRS["features"]]
    trainer = band_split.BandSplitTrainer(raw, features, cam, lrs, rank, world, row_weights=weights)
    y0, y1 = trainer.y0, trainer.y1
    gen = torch.Generator().manual_seed(7)
    gt_host = torch.randint(0, 256, (H, W, 3), dtype=torch.uint8, generator=gen).pin_memory()
    gt_dev = gt_host.to(device).float() / 255.0
    fgen = torch.Generator(device=device).manual_seed(11 + rank)
    feature_grad = torch.rand(y1 - y0, W, C, generator=fgen, device=device) / (H * W)

    for _ in range(args.warmup):
        trainer.step(gt_dev, feature_grad)
    torch.cuda.synchronize()

    def timed(e2e: bool, record_calls: bool):
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        timer.active = record_calls
        launches0 = native_launches()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            gt = (gt_host.to(device, non_blocking=True).float() / 255.0) if e2e else gt_dev
            loss = trainer.step(gt, feature_grad)
            if e2e:
                loss.item()
        end.record()
        torch.cuda.synchronize()
        timer.active = False
        timed.launches = native_launches() - launches0
        ms = start.elapsed_time(end)
        if dist is not None:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        return ms

    clocks = ClockSampler(int(str(device).split(":")[-1]) if ":" in str(device) else 0)
    clocks.start()
    trainer.timer.enabled = True
    ms = timed(e2e=False, record_calls=True)
    trainer.timer.enabled = False
    phases = {k: v / args.steps for k, v in trainer.timer.totals().items()}
    launches = timed.launches
    clock_info = clocks.stop()
    calls, counts = timer.totals_ms(), timer.counts()
    band_sizes = torch.tensor([[trainer.band_gaussians, trainer.fetched_rows]], device=device)
    if dist is not None:
        gathered = [torch.zeros_like(band_sizes) for _ in range(world)]
        dist.all_gather(gathered, band_sizes)
        band_sizes = torch.cat(gathered)
    all_phases = [phases]
    if dist is not None:
        all_phases = [None] * world
        dist.all_gather_object(all_phases, phases)
    ms_e2e = timed(e2e=True, record_calls=False)
    if rank == 0:
        line = {
            "metric": METRIC, "value": args.steps / (ms / 1000.0), "unit": "views/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "ms_per_view": ms / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32 (feature contractions in split bf16: hi*hi + hi*lo + lo*hi, fp32 accumulate)",
            "data": "synthetic (seeded config-4 distribution)",
            "config": {"workload": "config4: one 1920x1080 view split by tile rows, full fwd+bwd+Adam step",
                       "gaussians": s.n, "channels": C, "parallelism": f"tile-row bands x{world}",
                       "row_owners": args.row_owners if world > 1 else "one rank",
                       "band_weights": args.band_weights,
                       "bands": trainer.bands, "l2": "inputs larger than L2 (feature table "
                       f"{s.n * C * 4 / 1e9:.1f} GB)"},
            "call_ms_per_step": {k: v / args.steps for k, v in sorted(calls.items(), key=lambda kv: -kv[1])},
            "phase_ms_per_step": all_phases,
            "band_gaussians": [b[0] for b in band_sizes.tolist()],
            "fetched_feature_rows": [b[1] for b in band_sizes.tolist()],
            "gpu_launches": launches, "clocks": clock_info,
            "e2e": {"value": args.steps / (ms_e2e / 1000.0), "unit": "views/s",
                    "h2d_bytes_per_step": H * W * 3, "d2h_bytes_per_step": 4},
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def native_launches():
    from hds_b200 import native

    return native.lib.hds_launch_count()


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
    if args.split == "rows":
        run_band_split(args, device, rank, world, dist, timer)
        return
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
    per_view = {k: 1 for k in calls}
    stages = rooflines(calls, counts, per_view, stats, args.channels, n, peaks, world)
    dominant = max(stages, key=lambda k: stages[k]["ms"])
    roof = dict(stages[dominant])
    roof["kernel"] = dominant + " (" + ", ".join(c for c in STAGES[dominant] if c in calls) + ")"
    roof["traffic"] = None
    for call in STAGES[dominant]:
        fit = TRAFFIC_FIT.get((call, args.channels))
        if fit is not None and call in calls:
            roof["traffic"] = fit[0] + fit[1] * stats["visited"]
            roof["traffic_source"] = (f"a + b V (V = {stats['visited']} visited pairs) fitted to two small one-pass "
                                      f"captures, {fit[2]}")
    line = {
        "metric": METRIC, "value": value, "unit": "views/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "ms_per_view": ms / (args.steps * args.views),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 (feature contractions in split bf16: hi*hi + hi*lo + lo*hi, fp32 accumulate)",
        "data": DATA, "config": bench_config(args, world),
        "roofline": roof,
        "rooflines": stages,
        "call_ms_per_step": {k: v / args.steps for k, v in sorted(calls.items(), key=lambda kv: -kv[1])},
        "gpu_launches": launches,
        "tile_stats": stats,
        "clocks": clock_info,
        "e2e": e2e,
    }
    if world == 1 and not args.no_sweep:
        line["sweep"] = harness_sweep(args, device, timer, peaks)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args)
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

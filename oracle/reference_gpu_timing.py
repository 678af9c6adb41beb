"""Times the reference's own CUDA extension (built into oracle/_ref/) and this library on the same
B200, in the reference benchmark's scope (bench/harness.py:59-66, 133-177): projection of the
gaussians, then rasterize with features (colours as a leaf), forward and backward timed
separately, each the median of 50 runs after 10 warm-ups, bracketed by CUDA events.

Both implementations run through the same two-pass autograd glue, a restatement of the
reference's RasterizeGaussians / ProjectGaussians (rasterizer/__init__.py:57-165,
projection.py:25-93).  This library also runs through its own autograd path, which renders RGB and
features in one walk.  Before timing, the outputs must agree within the parity tolerances (as the
harness gates, harness.py:201-210).

    python oracle/reference_gpu_timing.py [--channels 32 64 128 256 512] [--gaussians 1180000]

Prints one JSON object per channel count.  Like everything under oracle/, this is test
infrastructure: it runs the reference's own build as the GPU bar this library is compared with.
"""
from __future__ import annotations

import argparse
import json
import statistics
import sys
import time
from pathlib import Path

import torch
import torch.nn.functional as F

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO / "high-dimensional-splatting_b200"))
sys.path.insert(0, str(REPO / "oracle"))

import build_ref  # noqa: E402
from hds_b200 import gaussian_rasterizer as ours  # noqa: E402
from hds_b200 import scenes  # noqa: E402
from hds_b200.rasterizer import rasterize as ours_fused  # noqa: E402
from hds_b200.projection import project_gaussians as ours_project  # noqa: E402

NEAR_PLANE, LOW_PASS, FOV_SCALE = 0.2, 0.3, 1.3


def two_pass(module):
    class Project(torch.autograd.Function):
        @staticmethod
        def forward(ctx, means, scales, quats, opacities, w2c, fx, fy, cx, cy, width, height):
            out = module.project_gaussians(means.contiguous(), scales.contiguous(), quats.contiguous(),
                                           opacities.detach().contiguous(), w2c, fx, fy, cx, cy, width, height,
                                           NEAR_PLANE, LOW_PASS, FOV_SCALE)
            ctx.save_for_backward(means, scales, quats, w2c)
            ctx.cam = (fx, fy, cx, cy, width, height)
            ctx.mark_non_differentiable(out[1], out[2])
            return out

        @staticmethod
        def backward(ctx, gm2, gd, gr, gcon):
            means, scales, quats, w2c = ctx.saved_tensors
            g = module.project_gaussians_backward(gm2.contiguous(), gcon.contiguous(), means.contiguous(),
                                                  scales.contiguous(), quats.contiguous(), w2c, *ctx.cam, NEAR_PLANE,
                                                  LOW_PASS, FOV_SCALE)
            return (*g, None, None, None, None, None, None, None, None)

    class Raster(torch.autograd.Function):
        @staticmethod
        def forward(ctx, means2D, depths, radii, conics, colors, opacities, background, features, width, height):
            image, T, nc, values, ranges, conic, co = module.rasterize(
                means2D.contiguous(), depths.contiguous(), radii.contiguous(), conics.contiguous(),
                colors.contiguous(), opacities.contiguous(), background, width, height)
            fimg, fT, fnc = module.rasterize_features(features, means2D.contiguous(), conic, co, values, ranges,
                                                      width, height)
            ctx.save_for_backward(means2D, conic, co, values, ranges, T, nc, background, features, fT, fnc)
            ctx.size = (width, height)
            return image, fimg

        @staticmethod
        def backward(ctx, gimg, gf):
            means2D, conic, co, values, ranges, T, nc, bg, features, fT, fnc = ctx.saved_tensors
            w, h = ctx.size
            gm, gc, gcol, go = module.rasterize_backward(gimg.contiguous(), means2D.contiguous(), conic, co, values,
                                                        ranges, T, nc, bg, w, h)
            gfeat, fm, fc, fo = module.rasterize_features_backward(gf.contiguous(), features, means2D.contiguous(),
                                                                   conic, co, values, ranges, fT, fnc, w, h,
                                                                   min(features.shape[1], 128))
            return gm + fm, None, None, gc + fc, gcol, go + fo, None, gfeat, None, None

    def render(leaves, cam):
        m2, d, r, c = Project.apply(leaves["means"], leaves["scales"], F.normalize(leaves["quats"], dim=-1),
                                    leaves["opacities"][:, None], cam.world_to_camera, cam.fx, cam.fy, cam.cx,
                                    cam.cy, cam.width, cam.height)
        bg = torch.zeros(3, device=m2.device)
        return Raster.apply(m2, d, r, c, leaves["colors"], leaves["opacities"][:, None], bg, leaves["features"],
                            cam.width, cam.height)

    return render


def render_ours_fused(leaves, cam):
    m2, d, r, c = ours_project(leaves["means"], leaves["scales"], F.normalize(leaves["quats"], dim=-1),
                               leaves["opacities"][:, None], cam.world_to_camera, cam.fx, cam.fy, cam.cx, cam.cy,
                               cam.width, cam.height)
    return ours_fused(m2, d, r, c, leaves["colors"], leaves["opacities"][:, None], cam.width, cam.height,
                      features=leaves["features"])


def time_ms(fn, before=None, iters=50, warmup=10):
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


def measure(render, inputs, cam):
    leaves = {k: v.clone().requires_grad_(True) for k, v in inputs.items() if not k.startswith("grad_")}
    state = {}

    def fwd():
        state["out"] = render(leaves, cam)

    def bwd():
        torch.autograd.backward(state["out"], [inputs["grad_image"], inputs["grad_feature_image"]])

    def reset():
        for leaf in leaves.values():
            leaf.grad = None
        fwd()

    f = time_ms(fwd)
    b = time_ms(bwd, before=reset)
    reset()
    bwd()
    return f, b, [o.detach() for o in state["out"]], {k: v.grad for k, v in leaves.items()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--channels", type=int, nargs="+", default=[32, 64, 128, 256, 512])
    ap.add_argument("--gaussians", type=int, default=1_180_000)
    args = ap.parse_args()
    ref = build_ref.load_built()
    dev = torch.device("cuda")
    for C in args.channels:
        s = scenes.config1(0, n=args.gaussians, channels=C)
        cam = s.cameras[0].to(dev)
        g = torch.Generator(device="cpu").manual_seed(0)
        inputs = {"means": s.means.to(dev), "scales": s.scales.to(dev), "quats": s.quats.to(dev),
                  "opacities": s.opacities[:, 0].contiguous().to(dev), "colors": torch.rand(s.n, 3, generator=g).to(dev),
                  "features": s.features.to(dev),
                  "grad_image": torch.rand(cam.height, cam.width, 3, generator=g).to(dev),
                  "grad_feature_image": torch.rand(cam.height, cam.width, C, generator=g).to(dev)}
        rows = {}
        results = {}
        for label, render in (("reference", two_pass(ref)), ("ours_two_pass", two_pass(ours)),
                              ("ours_fused", render_ours_fused)):
            f, b, outs, grads = measure(render, inputs, cam)
            rows[label] = {"fwd_ms": f, "bwd_ms": b, "fwd_bwd_ms": f + b}
            results[label] = (outs, grads)
            del outs, grads
        # Agreement gate (outputs of the reference vs this library).
        (ro, rg), (oo, og) = results["reference"], results["ours_fused"]
        agree = {"image_max_abs": (ro[0] - oo[0]).abs().max().item(),
                 "feature_max_abs": (ro[1] - oo[1]).abs().max().item(),
                 "feature_p99_abs": torch.quantile((ro[1] - oo[1]).abs().flatten()[:2**24].float(), 0.99).item()}
        for k in rg:
            scale = rg[k].abs().max().item()
            agree[f"grad_{k}_max_rel"] = ((rg[k] - og[k]).abs().max().item() / scale) if scale > 0 else 0.0
        print(json.dumps({"channels": C, "gaussians": args.gaussians, "view": f"{cam.width}x{cam.height}",
                          "timings": rows, "agreement": agree,
                          "speedup_fwd_bwd": rows["reference"]["fwd_bwd_ms"] / rows["ours_fused"]["fwd_bwd_ms"]}),
              flush=True)
        del results, inputs
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()

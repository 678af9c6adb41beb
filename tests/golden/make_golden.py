"""Writes the golden fixtures in tests/golden/ from the reference's own CPU code.

Run in a container that holds the reference checkout (it is not needed anywhere else):

    python tests/golden/make_golden.py /path/to/high-dimensional-splatting [--only model_init,densify]

It imports, from the reference:
  * tests/oracle.py::rasterize_reference       -- the fp64 dense blend (forward; autograd = backward)
  * tests/test_sh.py::eval_sh_reference        -- the term-by-term SH reference
  * gaussian_splatting/utils/loss.py::ssim     -- the torch SSIM path (CPU tensors take it)
  * gaussian_splatting/utils/gaussian.py::GaussianModel -- the point-cloud initialisation (model_init.npz) and
    densify_and_prune with its Adam surgery (densify.npz; torch.normal's draws recorded;
    its module imports pycolmap through utils/dataset.py, which is stubbed for the import since the
    initialisation does not use it)
and runs them on seeded inputs.  The 2-D inputs of the projected scenes come from the oracle's
projection (oracle/hds_oracle.c), since the reference has no CPU projection.  The fixtures hold
inputs and reference outputs; tests/test_oracle_golden.py checks the oracle against them.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "oracle"))
sys.path.insert(0, str(REPO / "high-dimensional-splatting_b200"))

import oracle  # noqa: E402
from hds_b200 import scenes  # noqa: E402

BACKGROUND = np.array([0.3, 0.5, 0.7], np.float32)


def load_reference(root: Path):
    sys.path.insert(0, str(root))
    from tests.oracle import rasterize_reference  # type: ignore
    from tests.test_sh import eval_sh_reference  # type: ignore
    from gaussian_splatting.utils.loss import ssim, _window  # type: ignore
    return rasterize_reference, eval_sh_reference, ssim, _window


def seeded_uniform(seed: int, shape) -> np.ndarray:
    """U[0, 1) float32 from numpy's PCG64, reproducible on every platform."""
    return np.random.default_rng(seed).random(shape, dtype=np.float32)


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def reference_raster(rasterize_reference, inputs, width, height, background, grad_image, features=None,
                     grad_features=None):
    """Forward and autograd backward of the reference oracle on one 2-D scene."""
    means2D, depths, radii, conics, colors, opacities = (t(x) for x in inputs)
    out = {}
    leaves = [x.clone().requires_grad_(True) for x in (means2D, conics, colors, opacities)]
    image = rasterize_reference(leaves[0], depths, radii, leaves[1], leaves[2], leaves[3], width, height,
                                t(background))
    image.backward(t(grad_image))
    out["image"] = image.detach().numpy()
    for name, leaf in zip(("means2D", "conics", "colors", "opacities"), leaves):
        out[f"grad_{name}"] = leaf.grad.numpy()
    if features is not None:
        leaves = [x.clone().requires_grad_(True) for x in (means2D, conics, t(features), opacities)]
        feat = rasterize_reference(leaves[0], depths, radii, leaves[1], leaves[2], leaves[3], width, height)
        feat.backward(t(grad_features))
        out["feature_image"] = feat.detach().numpy()
        for name, leaf in zip(("means2D", "conics", "features", "opacities"), leaves):
            out[f"feat_grad_{name}"] = leaf.grad.numpy()
    return out


def projected(scene_means, scales, quats, opacities, cam):
    return oracle.project_forward(scene_means, scales, quats, opacities, cam.world_to_camera.numpy(), cam.fx, cam.fy,
                                  cam.cx, cam.cy, cam.width, cam.height)


def main(root: Path) -> None:
    rasterize_reference, eval_sh_reference, ssim, _window = load_reference(root)
    torch.set_num_threads(8)
    rng = np.random.default_rng(1234)

    # 1. The reference tests' scene distribution, projected through an identity camera.
    width, height, n = 64, 48, 1500
    g = scenes.reference_test_scene(0, n)
    cam = scenes.identity_camera(width, height)
    m2, dep, rad, con = projected(g["means"].numpy(), g["scales"].numpy(), g["quats"].numpy(),
                                  g["opacities"].numpy(), cam)
    colors, opac = g["colors"].numpy(), g["opacities"].numpy()
    features = rng.random((n, 32), dtype=np.float32)
    grad_image = rng.random((height, width, 3), dtype=np.float32)
    grad_features = rng.random((height, width, 32), dtype=np.float32)
    inputs = (m2, dep, rad, con, colors, opac)
    ref = reference_raster(rasterize_reference, inputs, width, height, BACKGROUND, grad_image, features,
                           grad_features)
    np.savez_compressed(HERE / "raster_ref_scene.npz", width=width, height=height, means2D=m2, depths=dep, radii=rad,
                        conics=con, colors=colors, opacities=opac, background=BACKGROUND, features=features,
                        grad_image=grad_image, grad_features=grad_features, **ref)

    # 2. Config 0 (4,096 gaussians, 128x96, C = 32, SH degree 3 colours).
    s = scenes.config0(0, channels=32)
    cam = s.cameras[0]
    m2, dep, rad, con = projected(s.means.numpy(), s.scales.numpy(), s.quats.numpy(), s.opacities.numpy(), cam)
    dirs = torch.nn.functional.normalize(s.means - cam.center, dim=-1)
    sh = torch.cat([s.sh_dc, s.sh_rest], dim=1)
    colors = eval_sh_reference(sh.double(), dirs.double(), 3, t(rad)).float().numpy()
    opac = s.opacities.numpy()
    feats = s.features.numpy()
    # The gradient images are regenerated from these seeds by the tests (numpy PCG64 is portable).
    grad_image = seeded_uniform(101, (cam.height, cam.width, 3))
    grad_features = seeded_uniform(102, (cam.height, cam.width, 32))
    inputs = (m2, dep, rad, con, colors, opac)
    ref = reference_raster(rasterize_reference, inputs, cam.width, cam.height, BACKGROUND, grad_image, feats,
                           grad_features)
    np.savez_compressed(HERE / "raster_config0.npz", width=cam.width, height=cam.height, means2D=m2, depths=dep,
                        radii=rad, conics=con, colors=colors, opacities=opac, background=BACKGROUND, features=feats,
                        grad_image_seed=101, grad_features_seed=102, **ref)

    # 3. The flat edge-case scenes of the reference's tests/test_render.py:137-225.
    def flat(means, depths, sigmas, opacities, seed):
        k = len(depths)
        sigma = np.asarray(sigmas, np.float32)
        r = np.random.default_rng(seed)
        return (np.asarray(means, np.float32), np.asarray(depths, np.float32), np.ones(k, np.float32),
                np.stack([sigma ** -2, np.zeros_like(sigma), sigma ** -2], -1).astype(np.float32),
                r.random((k, 3), dtype=np.float32), np.asarray(opacities, np.float32)[:, None])

    r = np.random.default_rng(11)
    dense_means = (r.random((2000, 2), dtype=np.float32) * 16).tolist()
    dense_depths = (1 + r.random(2000, dtype=np.float32)).tolist()
    cases = {
        "depth_ties": (flat([[7.5, 8.5], [9.5, 8.5]], [2.0, 2.0], [3.0, 3.0], [0.7, 0.7], 2), 16, 16),
        "min_alpha": (flat([[4.5, 4.5], [12.5, 4.5]], [1.0, 1.0], [0.5, 0.5], [1.01 / 255, 0.99 / 255], 3), 16, 8),
        "max_alpha": (flat([[8.5, 8.5]], [1.0], [2.0], [1.0], 4), 16, 16),
        "t_floor": (flat([[8.5, 8.5]] * 50, [1.0 + i for i in range(50)], [4.0] * 50, [0.9] * 50, 5), 16, 16),
        "dense_tile": (flat(dense_means, dense_depths, [12.0] * 2000, [0.02] * 2000, 6), 16, 16),
    }
    flat_out = {}
    for name, (inputs, w, h) in cases.items():
        k = len(inputs[1])
        feats = r.random((k, 32), dtype=np.float32)
        gi = r.random((h, w, 3), dtype=np.float32)
        gf = r.random((h, w, 32), dtype=np.float32)
        ref = reference_raster(rasterize_reference, inputs, w, h, BACKGROUND, gi, feats, gf)
        for key, val in zip(("means2D", "depths", "radii", "conics", "colors", "opacities"), inputs):
            flat_out[f"{name}__{key}"] = val
        flat_out.update({f"{name}__features": feats, f"{name}__grad_image": gi, f"{name}__grad_features": gf,
                         f"{name}__size": np.array([w, h])})
        flat_out.update({f"{name}__{key}": val for key, val in ref.items()})
    np.savez_compressed(HERE / "raster_flat.npz", background=BACKGROUND, **flat_out)

    # 4. Spherical harmonics: forward at degrees 0-3, autograd dirs/SH gradients, and 3 Adam steps.
    gsh = torch.Generator().manual_seed(5)
    n = 512
    sh = torch.randn(n, 16, 3, generator=gsh) * 0.5
    dirs = torch.nn.functional.normalize(torch.randn(n, 3, generator=gsh), dim=-1)
    radii = (torch.rand(n, generator=gsh) > 0.1).float()
    grad_rgb = torch.randn(n, 3, generator=gsh)
    out = {"sh": sh.numpy(), "dirs": dirs.numpy(), "radii": radii.numpy(), "grad_rgb": grad_rgb.numpy()}
    for degree in range(4):
        s64 = sh.double().requires_grad_(True)
        d64 = dirs.double().requires_grad_(True)
        rgb = eval_sh_reference(s64, d64, degree, radii)
        rgb.backward(grad_rgb.double())
        out[f"rgb_{degree}"] = rgb.detach().float().numpy()
        out[f"grad_sh_{degree}"] = s64.grad.float().numpy()
        out[f"grad_dirs_{degree}"] = d64.grad.float().numpy()
    dc = torch.nn.Parameter(sh[:, :1].clone())
    rest = torch.nn.Parameter(sh[:, 1:].clone())
    adam = torch.optim.Adam([{"params": [dc], "lr": 0.0025}, {"params": [rest], "lr": 0.0025 / 20}], eps=1e-15,
                            foreach=False)
    steps = []
    for _ in range(3):
        gr = torch.randn(n, 3, generator=gsh)
        steps.append(gr.numpy())
        eval_sh_reference(torch.cat([dc, rest], dim=1), dirs, 3, radii).backward(gr)
        adam.step()
        adam.zero_grad(set_to_none=True)
    out["adam_grad_rgb"] = np.stack(steps)
    out["adam_dc"], out["adam_rest"] = dc.detach().numpy(), rest.detach().numpy()
    for key, p in (("dc", dc), ("rest", rest)):
        st = adam.state[p]
        out[f"adam_m_{key}"] = st["exp_avg"].numpy()
        out[f"adam_v_{key}"] = st["exp_avg_sq"].numpy()
    np.savez_compressed(HERE / "sh.npz", **out)

    # 5. SSIM on the reference test's sizes (tests/test_ssim.py:17-31), torch path in fp64.
    out = {"window": _window(11, 1.5, torch.device("cpu"), torch.float32)[0, 0].numpy()}
    for (hh, ww) in [(64, 64), (37, 53), (11, 11)]:
        gs = torch.Generator().manual_seed(hh * ww)
        gt = torch.rand(hh, ww, 3, generator=gs)
        rendered = (gt + 0.1 * torch.randn(hh, ww, 3, generator=gs)).clamp(0, 1)
        x = rendered.double().requires_grad_(True)
        val = ssim(x, gt.double())
        val.backward()
        out[f"{hh}x{ww}_rendered"] = rendered.numpy()
        out[f"{hh}x{ww}_gt"] = gt.numpy()
        out[f"{hh}x{ww}_ssim"] = np.float64(val.item())
        out[f"{hh}x{ww}_grad"] = x.grad.numpy()
    np.savez_compressed(HERE / "ssim.npz", **out)
    print("fixtures written to", HERE)


def model_init_fixture(root: Path) -> None:
    """GaussianModel(point_cloud, device='cpu').params of a seeded cloud of 500 points."""
    import types

    sys.path.insert(0, str(root))
    stub = types.ModuleType("pycolmap")
    stub.Image = stub.Reconstruction = object  # only used in annotations of the dataset loader
    sys.modules.setdefault("pycolmap", stub)
    from gaussian_splatting.utils.dataset import PointCloud  # type: ignore
    from gaussian_splatting.utils.gaussian import GaussianModel  # type: ignore

    rng = np.random.default_rng(77)
    points = rng.normal(0.0, 1.5, (500, 3)).astype(np.float32)
    points[7] = points[3]  # a duplicate point: zero distance to its nearest neighbour (the 1e-7 clamp)
    colors = rng.random((500, 3), dtype=np.float32)
    model = GaussianModel(PointCloud(points=points, colors=colors), device="cpu")
    out = {"points": points, "colors": colors}
    out.update({f"param_{k}": v.detach().numpy() for k, v in model.params.items()})
    np.savez_compressed(HERE / "model_init.npz", **out)
    print("model_init.npz written to", HERE)


def densify_fixture(root: Path) -> None:
    """GaussianModel.densify_and_prune (utils/gaussian.py:162-296) on a seeded CPU model whose sizes,
    opacities and accumulated 2-D gradients straddle every threshold, with an Adam state from one
    step; torch.normal's draws for the split children are recorded so that the device version can
    be fed the same offsets."""
    import types

    sys.path.insert(0, str(root))
    stub = types.ModuleType("pycolmap")
    stub.Image = stub.Reconstruction = object
    sys.modules.setdefault("pycolmap", stub)
    from gaussian_splatting.config import TrainingParams  # type: ignore
    from gaussian_splatting.utils.dataset import PointCloud  # type: ignore
    from gaussian_splatting.utils.gaussian import GaussianModel  # type: ignore

    torch.manual_seed(5)
    rng = np.random.default_rng(88)
    n = 600
    points = rng.normal(0.0, 1.0, (n, 3)).astype(np.float32)
    colors = rng.random((n, 3), dtype=np.float32)
    model = GaussianModel(PointCloud(points=points, colors=colors), device="cpu")
    params = TrainingParams()
    extent = 2.0
    with torch.no_grad():
        # scales around percent_dense * extent (0.02) and 0.1 * extent; opacities around min_opacity.
        model.params["scales"].copy_(torch.from_numpy(rng.normal(np.log(0.02), 1.2, (n, 3)).astype(np.float32)))
        model.params["quats"].copy_(torch.from_numpy(rng.normal(0, 1, (n, 4)).astype(np.float32)))
        model.params["opacities"].copy_(torch.from_numpy(rng.normal(-4.0, 2.0, (n, 1)).astype(np.float32)))
        model.params["sh_rest"].copy_(torch.from_numpy(rng.normal(0, 0.1, (n, 15, 3)).astype(np.float32)))
    optimizer = torch.optim.Adam(model.get_optimizer_params(params, extent), eps=1e-15)
    for group in optimizer.param_groups:
        p = group["params"][0]
        p.grad = torch.from_numpy(rng.normal(0, 1e-3, tuple(p.shape)).astype(np.float32))
    optimizer.step()
    model.means2D_grad_accum = torch.from_numpy(rng.random((n, 1), dtype=np.float32) * 4e-3)
    model.denom = torch.from_numpy(rng.integers(0, 12, (n, 1)).astype(np.float32))
    model.max_radii2D = torch.from_numpy(rng.random(n, dtype=np.float32) * 40.0)
    before = {f"in_param_{k}": v.detach().numpy().copy() for k, v in model.params.items()}
    for group in optimizer.param_groups:
        st = optimizer.state[group["params"][0]]
        before[f"in_m_{group['name']}"] = st["exp_avg"].numpy().copy()
        before[f"in_v_{group['name']}"] = st["exp_avg_sq"].numpy().copy()
    stats = {"in_grad_accum": model.means2D_grad_accum.numpy().copy(), "in_denom": model.denom.numpy().copy(),
             "in_max_radii2D": model.max_radii2D.numpy().copy()}
    drawn = []
    real_normal = torch.normal

    def recording_normal(*a, **k):
        out = real_normal(*a, **k)
        drawn.append(out.detach().clone())
        return out

    torch.normal = recording_normal
    try:
        model.densify_and_prune(optimizer, params, extent, max_screen_size=params.max_screen_size)
    finally:
        torch.normal = real_normal
    out = {**before, **stats, "extent": np.float32(extent), "normals": drawn[0].numpy()}
    out.update({f"out_param_{k}": v.detach().numpy() for k, v in model.params.items()})
    for group in optimizer.param_groups:
        st = optimizer.state[group["params"][0]]
        out[f"out_m_{group['name']}"] = st["exp_avg"].numpy()
        out[f"out_v_{group['name']}"] = st["exp_avg_sq"].numpy()
    np.savez_compressed(HERE / "densify.npz", **out)
    print("densify.npz written to", HERE, {k: v.shape for k, v in out.items() if k.startswith("out_param")})


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    root = Path(args[0] if args else "/root/reference")
    if "--only" in sys.argv:
        parts = sys.argv[sys.argv.index("--only") + 1].split(",")
        if "model_init" in parts:
            model_init_fixture(root)
        if "densify" in parts:
            densify_fixture(root)
    else:
        main(root)
        model_init_fixture(root)
        densify_fixture(root)

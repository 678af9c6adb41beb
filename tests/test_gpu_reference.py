"""This library against the reference's own CUDA extension (built from its sources into oracle/_ref/
by oracle/build_ref.py), on identical inputs.

The reference compiles with --use_fast_math (hardware exp/log approximations, contracted FMAs), so
agreement is within tolerance rather than bit-exact:
  * projection: within 2e-5 relative except a few in 1e5 conics (none beyond 1e-3), visibility equal
    except for a handful at the cull edge;
  * RGB image: within 1e-5 except pixels where a pair sits on the MIN_ALPHA / MIN_T cutoff (<= 0.1%);
  * features: both TF32 (the reference also rounds with cvt.rna), within 1e-3;
  * gradients: helpers.assert_grads_close (1e-4 of the largest gradient).
"""
import numpy as np
import pytest

from helpers import FEATURE_ATOL, assert_close_fastmath, assert_grads_close, assert_grads_close_fastmath
from scenes_np import config_scene, reference_scene

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

BACKGROUND = np.array([0.3, 0.5, 0.7], np.float32)


@pytest.fixture(scope="module")
def mods():
    import build_ref

    if build_ref.built() is None:
        pytest.skip("the reference extension is not built (oracle/build_ref.py needs the reference checkout)")
    from hds_b200 import gaussian_rasterizer

    return build_ref.load_built(), gaussian_rasterizer


def cuda(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]


def host(t):
    return t.detach().cpu().numpy()


SCENES = {
    "reference_128x96": lambda: (reference_scene(0, 3000, 128, 96), 128, 96),
    "config1_20k": lambda: (lambda sc: (sc[0], sc[1].width, sc[1].height))(
        config_scene(__import__("hds_b200.scenes", fromlist=["config1"]).config1(0, n=20_000, channels=0))),
}


@pytest.mark.parametrize("which", ["config0", "config1"])
def test_projection_matches_reference(mods, which):
    from hds_b200 import scenes

    ref, ours = mods
    s = scenes.config0(0, channels=0) if which == "config0" else scenes.config1(0, n=50_000, channels=0)
    cam = s.cameras[0]
    t = cuda(s.means.numpy(), s.scales.numpy(), s.quats.numpy(), s.opacities.numpy(), cam.world_to_camera.numpy())
    args = (cam.fx, cam.fy, cam.cx, cam.cy, cam.width, cam.height, 0.2, 0.3, 1.3)
    a = [host(x) for x in ref.project_gaussians(*t, *args)]
    b = [host(x) for x in ours.project_gaussians(*t, *args)]
    vis_a, vis_b = a[2] > 0, b[2] > 0
    assert (vis_a != vis_b).mean() < 1e-3
    both = vis_a & vis_b
    for name, x, y in zip(("means2D", "depths", "radii", "conics"), a, b):
        x, y = x[both].astype(np.float64), y[both].astype(np.float64)
        # The conic inverts the 2x2 covariance: det = a*c - b*b cancels for elongated gaussians and
        # amplifies the reference's fast-math contractions, so a few in 1e5 exceed 2e-5 relative.
        diff, scale = np.abs(y - x), np.abs(x).max()
        bad = diff > 2e-5 * np.abs(x) + 1e-6 * scale
        assert bad.mean() <= 1e-4, f"{name}: {bad.sum()} of {bad.size} beyond 2e-5 relative"
        assert (diff <= 1e-3 * np.abs(x) + 1e-5 * scale).all(), f"{name}: worst difference {diff.max():.3e}"


@pytest.mark.parametrize("scene", list(SCENES))
def test_rasterize_matches_reference(mods, scene):
    ref, ours = mods
    inputs, w, h = SCENES[scene]()
    t = cuda(*inputs, BACKGROUND)
    ra = ref.rasterize(*t, w, h)
    ob = ours.rasterize(*t, w, h)
    assert abs(ra[3].numel() - ob[3].numel()) <= max(2, 1e-3 * ra[3].numel()), "pair counts differ"
    assert_close_fastmath(host(ob[0]), host(ra[0]), 1e-5, "image")
    assert (host(ob[2]) != host(ra[2])).mean() < 1e-3, "n_contrib differs"
    gi = torch.rand(h, w, 3, generator=torch.Generator(device="cuda").manual_seed(1), device="cuda")
    ga = ref.rasterize_backward(gi, t[0], ra[5], ra[6], ra[3], ra[4], ra[1], ra[2], t[6], w, h)
    gb = ours.rasterize_backward(gi, t[0], ob[5], ob[6], ob[3], ob[4], ob[1], ob[2], t[6], w, h)
    for name, x, y in zip(("means2D", "conics", "colors", "opacities"), ga, gb):
        assert_grads_close_fastmath(host(y), host(x), name)


@pytest.mark.parametrize("channels", [32, 128, 512])
@pytest.mark.parametrize("scene", list(SCENES))
def test_features_match_reference(mods, scene, channels):
    ref, ours = mods
    inputs, w, h = SCENES[scene]()
    t = cuda(*inputs, BACKGROUND)
    gen = torch.Generator(device="cuda").manual_seed(channels)
    feats = torch.rand(len(inputs[1]), channels, generator=gen, device="cuda")
    ra = ref.rasterize(*t, w, h)
    ob = ours.rasterize(*t, w, h)
    fa = ref.rasterize_features(feats, t[0], ra[5], ra[6], ra[3], ra[4], w, h)
    fb = ours.rasterize_features(feats, t[0], ob[5], ob[6], ob[3], ob[4], w, h)
    assert_close_fastmath(host(fb[0]), host(fa[0]), FEATURE_ATOL, "feature image")
    gf = torch.rand(h, w, channels, generator=gen, device="cuda")
    width = min(channels, 128)
    ga = ref.rasterize_features_backward(gf, feats, t[0], ra[5], ra[6], ra[3], ra[4], fa[1], fa[2], w, h, width)
    gb = ours.rasterize_features_backward(gf, feats, t[0], ob[5], ob[6], ob[3], ob[4], fb[1], fb[2], w, h, width)
    for name, x, y in zip(("features", "means2D", "conics", "opacities"), ga, gb):
        assert_grads_close_fastmath(host(y), host(x), name)


def test_sh_and_ssim_match_reference(mods, golden):
    ref, ours = mods
    g = golden("sh.npz")
    sh, dirs, radii = g["sh"], g["dirs"], g["radii"]
    dc, rest = np.ascontiguousarray(sh[:, :1]), np.ascontiguousarray(sh[:, 1:])
    t = cuda(dc, rest, dirs, radii)
    for degree in range(4):
        np.testing.assert_allclose(host(ours.eval_sh(*t[:3], degree, t[3])), host(ref.eval_sh(*t[:3], degree, t[3])),
                                   rtol=1e-5, atol=1e-6)
    s = golden("ssim.npz")
    a, b = cuda(s["64x64_rendered"], s["64x64_gt"])
    xa, xb = ref.ssim_forward(a, b), ours.ssim_forward(a, b)
    # The SSIM value, then its derivative maps.  The maps divide by (mu^2 + C1)(sigma^2 + C2), where
    # the reference's fast-math division differs by a few ulp: compare them against their scale.
    np.testing.assert_allclose(host(xb[0]), host(xa[0]), rtol=1e-4, atol=1e-6)
    for i, (x, y) in enumerate(zip(xa[1:], xb[1:])):
        assert_grads_close(host(y), host(x), f"ssim derivative map {i}")
    gm = torch.ones(1, device="cuda")
    assert_grads_close(host(ours.ssim_backward(gm, a, b, *xb[1:])), host(ref.ssim_backward(gm, a, b, *xa[1:])),
                       "ssim gradient")

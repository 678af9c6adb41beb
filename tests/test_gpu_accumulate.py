"""The in-place feature-gradient path (rasterizer.ACCUMULATE_INTO_LEAF_GRAD, backed by
hds_render_features_backward_accumulate) against the standard autograd path: two views accumulated
into a pre-allocated .grad give the same gradients for every leaf."""
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _grads(accumulate: bool, channels: int):
    """Two views' rasterizer gradients accumulated into pre-allocated .grad buffers.  The leaves are
    the rasterizer's own inputs (2-D means, conics, opacities, colours, features): the projection
    backward would amplify the float-atomic ordering noise of near-degenerate conics."""
    from hds_b200 import rasterizer, scenes
    from hds_b200.projection import project_gaussians

    s = scenes.config1(3, n=20_000, channels=channels)
    features = s.features.cuda().requires_grad_(True)
    opacities = s.opacities.cuda().requires_grad_(True)
    colors = torch.rand(s.n, 3, device="cuda", generator=torch.Generator(device="cuda").manual_seed(0),
                        requires_grad=True)
    views = []
    for cam in s.cameras[:2]:
        cam = cam.to("cuda")
        with torch.no_grad():
            m2, d, r, c = project_gaussians(s.means.cuda(), s.scales.cuda(), s.quats.cuda(), s.opacities.cuda(),
                                            cam.world_to_camera, cam.fx, cam.fy, cam.cx, cam.cy, cam.width,
                                            cam.height)
        views.append((cam, m2.requires_grad_(True), d, r, c.requires_grad_(True)))
    leaves = {"features": features, "opacities": opacities, "colors": colors}
    for t in leaves.values():
        t.grad = torch.zeros_like(t)
    g = torch.Generator(device="cuda").manual_seed(1)
    out = {}
    for i, (cam, m2, d, r, c) in enumerate(views):
        old = rasterizer.ACCUMULATE_INTO_LEAF_GRAD
        rasterizer.ACCUMULATE_INTO_LEAF_GRAD = accumulate
        try:
            img, fimg = rasterizer.rasterize(m2, d, r, c, colors, opacities, cam.width, cam.height,
                                             features=features)
        finally:
            rasterizer.ACCUMULATE_INTO_LEAF_GRAD = old
        gi = torch.rand(img.shape, device="cuda", generator=g)
        gf = torch.rand(fimg.shape, device="cuda", generator=g)
        torch.autograd.backward([img, fimg], [gi, gf])
        out[f"means2D_{i}"] = m2.grad.clone()
        out[f"conics_{i}"] = c.grad.clone()
    return {k: v.grad.clone() for k, v in leaves.items()} | out


@pytest.mark.parametrize("channels", [32, 512])
def test_accumulate_matches_autograd(channels):
    from helpers import assert_grads_close

    want = _grads(False, channels)
    got = _grads(True, channels)
    # Only the destination of dL/dfeatures differs; float atomics add in a different order on every
    # run, hence the suite's gradient bound.
    for k in want:
        assert_grads_close(got[k].cpu().numpy(), want[k].cpu().numpy(), k)
    f_err = (got["features"] - want["features"]).abs().max().item()
    assert f_err <= 1e-5 * want["features"].abs().max().item(), f"features: max |diff| {f_err:.3e}"


def test_accumulate_requires_matching_grad_buffer():
    from hds_b200 import gaussian_rasterizer as ext

    f = torch.zeros(10, 32, device="cuda")
    bad = torch.zeros(10, 64, device="cuda")
    with pytest.raises(RuntimeError, match="shaped like features"):
        ext.rasterize_features_backward_into(bad, torch.zeros(4, 4, 32, device="cuda"), f, None, None, None, None,
                                             None, None, None, 4, 4, 32)


def test_bucket_zero_async_clears_before_the_backward():
    """GradBucket.zero_async clears on a side stream; after ready() the current stream sees zeros, and
    gradients added afterwards land on the cleared buffer."""
    from hds_b200 import parallel

    params = [torch.randn(300_000, 3, device="cuda", requires_grad=True),
              torch.randn(1000, 16, device="cuda", requires_grad=True)]
    bucket = parallel.GradBucket(params)
    for _ in range(3):
        bucket.flat.fill_(7.0)
        bucket.zero_async()
        bucket.ready()
        (params[0].sum() + 2.0 * params[1].sum()).backward()
        assert torch.equal(params[0].grad, torch.ones_like(params[0]))
        assert torch.equal(params[1].grad, torch.full_like(params[1], 2.0))

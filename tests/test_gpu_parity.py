"""Stage-by-stage parity of the CUDA path (called through the C ABI) with the CPU oracle.

Bit-exact (np.array_equal): projection, SH colour and SH gradients, tile keys, sort order, tile
ranges, the RGB image, final transmittance, contributor counts, and SSIM (map, partials, gradient).
The forward kernels are compiled with --fmad=false and use the oracle's exact operation order.

Within tolerance:
  * feature images: split-bf16 tensor-core contraction (hi*hi + hi*lo + lo*hi).  Against the exact
    FP32 oracle within the north star's 1e-3 absolute, for features drawn U[0, 1) (the reference
    tests' distribution) and N(0, 1) (the benchmark configs'); against the oracle that forms the
    same split products (exact, double sums) within 1e-5 * max(1, max|f|), which catches any
    operand-layout error.
  * gradients: accumulated with float atomics in any order; every entry within 1e-4 of the tensor's
    largest gradient (helpers.assert_grads_close) against the oracle's double sums.  Forward and
    backward compute every pair's alpha with the same operations as the oracle, so no pair changes
    side of the MIN_ALPHA cutoff between them.
"""
import numpy as np
import pytest

import oracle
from helpers import FEATURE_ATOL, assert_close_abs, assert_grads_close
from scenes_np import GOLDEN_FLAT_CASES, SIZE_EXAMPLES, config_scene, golden_case, reference_scene

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

CASES = ["raster_ref_scene", "raster_config0", *GOLDEN_FLAT_CASES, *[f"size{i}" for i in range(len(SIZE_EXAMPLES))],
         "config1_20k"]
BACKGROUND = np.array([0.3, 0.5, 0.7], np.float32)
_cache = {}


@pytest.fixture(scope="module")
def ext():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from hds_b200 import gaussian_rasterizer

    return gaussian_rasterizer


def cuda(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]


def host(t):
    return t.detach().cpu().numpy()


def case(name, golden):
    if name in _cache:
        return _cache[name]
    if name.startswith("size"):
        seed, n, w, h = SIZE_EXAMPLES[int(name[4:])]
        out = (reference_scene(seed, n, w, h), w, h)
    elif name == "config1_20k":
        from hds_b200 import scenes

        inputs, cam = config_scene(scenes.config1(0, n=20_000, channels=0))
        out = (inputs, cam.width, cam.height)
    else:
        inputs, w, h, _ = golden_case(golden, name)
        out = (inputs, w, h)
    _cache[name] = out
    return out


def features_for(n, channels, seed=0, dist="uniform"):
    rng = np.random.default_rng(1000 + channels + seed)
    if dist == "normal":
        return rng.standard_normal((n, channels), dtype=np.float32)
    return rng.random((n, channels), dtype=np.float32)


@pytest.mark.parametrize("name", CASES)
def test_binning_bit_exact(ext, golden, name):
    (m2, dep, rad, con, col, opac), w, h = case(name, golden)
    _, keys, values, ranges = oracle.bin_gaussians(m2, dep, rad, con, opac, w, h)
    g_keys, g_values, g_ranges = ext.bin_gaussians(*cuda(m2, dep, rad, con, opac), w, h)
    assert np.array_equal(host(g_keys).view(np.uint64), keys), "tile keys differ"
    assert np.array_equal(host(g_values), values), "sort order differs"
    assert np.array_equal(host(g_ranges), ranges), "tile ranges differ"


@pytest.mark.parametrize("name", CASES)
def test_rgb_forward_bit_exact(ext, golden, name):
    inputs, w, h = case(name, golden)
    m2, dep, rad, con, col, opac = inputs
    want = oracle.rasterize(*inputs, w, h, background=BACKGROUND)
    image, final_T, n_contrib, values, ranges, conic, co = ext.rasterize(*cuda(*inputs, BACKGROUND), w, h)
    assert np.array_equal(host(image), want["image"]), "image differs"
    assert np.array_equal(host(final_T), want["final_T"]), "final_T differs"
    assert np.array_equal(host(n_contrib), want["n_contrib"]), "n_contrib differs"


@pytest.mark.parametrize("dist", ["uniform", "normal"])
@pytest.mark.parametrize("channels", [32, 64, 128, 256, 512])
@pytest.mark.parametrize("name", ["raster_ref_scene", "raster_config0", "dense_tile", "t_floor", "size3", "size4",
                                  "config1_20k"])
def test_feature_forward(ext, golden, name, channels, dist):
    inputs, w, h = case(name, golden)
    m2, dep, rad, con, col, opac = inputs
    feats = features_for(len(dep), channels, dist=dist)
    want = oracle.rasterize(*inputs, w, h, background=BACKGROUND, features=feats)
    want_split = oracle.render_forward(want["ranges"], want["values"], m2, con, None, opac, w, h, features=feats,
                                       split_bf16=True)[3]
    t_in = cuda(*inputs, BACKGROUND)
    f = cuda(feats)[0]
    image, fimg, final_T, n_contrib, *_ = ext.rasterize_with_features(*t_in, f, w, h)
    from hds_b200.native import device_status

    assert device_status() == 0, "a bounded wait in the feature blend ran out"
    assert np.array_equal(host(image), want["image"]), "fused RGB differs"
    assert np.array_equal(host(final_T), want["final_T"]), "final_T differs"
    assert np.array_equal(host(n_contrib), want["n_contrib"]), "n_contrib differs"
    scale = max(1.0, float(np.abs(feats).max())) if feats.size else 1.0
    assert_close_abs(host(fimg), want_split, 1e-5 * scale, "feature image vs split-bf16 oracle")
    assert_close_abs(host(fimg), want["features"], FEATURE_ATOL, "feature image vs FP32 oracle")
    # The reference's two-pass API (rasterize then rasterize_features) gives the same image.
    _, _, _, values, ranges, conic, co = ext.rasterize(*t_in, w, h)
    fimg2, t2, c2 = ext.rasterize_features(f, t_in[0], conic, co, values, ranges, w, h)
    assert torch.equal(fimg2, fimg) and torch.equal(t2, final_T) and torch.equal(c2, n_contrib)


@pytest.mark.parametrize("name", CASES)
def test_rgb_backward(ext, golden, name):
    inputs, w, h = case(name, golden)
    m2, dep, rad, con, col, opac = inputs
    want = oracle.rasterize(*inputs, w, h, background=BACKGROUND)
    grad_image = np.random.default_rng(5).random((h, w, 3), dtype=np.float32)
    gm, gc, gcol, go, _ = oracle.render_backward(want["ranges"], want["values"], m2, con, col, opac, w, h,
                                                 want["final_T"], want["n_contrib"], grad_image=grad_image,
                                                 background=BACKGROUND)
    t_in = cuda(*inputs, BACKGROUND)
    _, final_T, n_contrib, values, ranges, conic, co = ext.rasterize(*t_in, w, h)
    got = ext.rasterize_backward(cuda(grad_image)[0], t_in[0], conic, co, values, ranges, final_T, n_contrib,
                                 t_in[6], w, h)
    for nm, g, wv in zip(("means2D", "conics", "colors", "opacities"), got, (gm, gc, gcol, go)):
        assert_grads_close(host(g), wv, nm)


@pytest.mark.parametrize("channels, slice_width", [(32, 32), (64, 64), (64, 32), (128, 128), (128, 64), (128, 32),
                                                   (256, 128), (256, 64), (512, 128), (512, 64)])
@pytest.mark.parametrize("name", ["raster_ref_scene", "raster_config0", "dense_tile", "size3", "config1_20k"])
def test_feature_backward(ext, golden, name, channels, slice_width):
    inputs, w, h = case(name, golden)
    m2, dep, rad, con, col, opac = inputs
    feats = features_for(len(dep), channels)
    grad_f = np.random.default_rng(9).random((h, w, channels), dtype=np.float32)
    want = oracle.rasterize(*inputs, w, h, background=BACKGROUND)
    gm, gc, _, go, gf = oracle.render_backward(want["ranges"], want["values"], m2, con, None, opac, w, h,
                                               want["final_T"], want["n_contrib"], features=feats,
                                               grad_features=grad_f)
    t_in = cuda(*inputs, BACKGROUND)
    _, final_T, n_contrib, values, ranges, conic, co = ext.rasterize(*t_in, w, h)
    got = ext.rasterize_features_backward(cuda(grad_f)[0], cuda(feats)[0], t_in[0], conic, co, values, ranges,
                                          final_T, n_contrib, w, h, slice_width)
    for nm, g, wv in zip(("features", "means2D", "conics", "opacities"), got, (gf, gm, gc, go)):
        assert_grads_close(host(g), wv, nm)


@pytest.mark.parametrize("channels, slice_width", [(256, 128), (256, 64), (512, 128), (512, 64)])
@pytest.mark.parametrize("name", ["raster_ref_scene", "dense_tile", "size3", "config1_20k"])
def test_feature_backward_cluster_kernel(ext, golden, monkeypatch, name, channels, slice_width):
    """256 and 512 channels on the four-block clusters (one walk per pixel, dot partials and weights
    exchanged through distributed shared memory), which HDS_FEATURE_BWD_CLUSTER=1 selects."""
    monkeypatch.setenv("HDS_FEATURE_BWD_CLUSTER", "1")
    test_feature_backward(ext, golden, name, channels, slice_width)


@pytest.mark.parametrize("channels, slice_width", [(256, 128), (512, 128), (512, 64)])
@pytest.mark.parametrize("name", ["raster_ref_scene", "dense_tile", "size3", "config1_20k"])
def test_feature_backward_one_block_kernel(ext, golden, monkeypatch, name, channels, slice_width):
    """256 and 512 channels on the one-block kernel (one walk per 128-channel slice), which
    HDS_FEATURE_BWD_CLUSTER=0 selects."""
    monkeypatch.setenv("HDS_FEATURE_BWD_CLUSTER", "0")
    test_feature_backward(ext, golden, name, channels, slice_width)


@pytest.mark.parametrize("channels", [256, 512])
@pytest.mark.parametrize("name", ["raster_ref_scene", "dense_tile", "config1_20k"])
@pytest.mark.parametrize("with_rgb", [True, False])
def test_fused_backward_cluster_kernel(ext, golden, monkeypatch, name, channels, with_rgb):
    monkeypatch.setenv("HDS_FEATURE_BWD_CLUSTER", "1")
    test_fused_backward(ext, golden, name, channels, with_rgb)


@pytest.mark.parametrize("helper", ["0", "2", "3", "7"])
@pytest.mark.parametrize("name", ["raster_ref_scene", "dense_tile", "size3", "config1_20k"])
@pytest.mark.parametrize("with_rgb", [True, False])
def test_fused_backward_cluster_helper_split(ext, golden, monkeypatch, name, helper, with_rgb):
    """At 512 channels the one-block kernel, on a second stream, takes every M-th half tile
    (HDS_FEATURE_BWD_HELPER=M) while the clusters take the rest; "0" runs the clusters alone.  Every
    split gives the oracle's gradients, the RGB terms included (the helper's first slice carries
    them)."""
    monkeypatch.setenv("HDS_FEATURE_BWD_HELPER", helper)
    test_fused_backward(ext, golden, name, 512, with_rgb)


@pytest.mark.parametrize("channels", [32, 128, 256, 512])
@pytest.mark.parametrize("name", ["raster_ref_scene", "raster_config0", "dense_tile", "size3", "config1_20k"])
@pytest.mark.parametrize("with_rgb", [True, False])
def test_fused_backward(ext, golden, name, channels, with_rgb, half_tile_lists=True):
    """hds_render_backward_fused: the RGB and feature backward in one walk, against the oracle run with
    both gradients at once (and with the feature terms alone)."""
    inputs, w, h = case(name, golden)
    m2, dep, rad, con, col, opac = inputs
    feats = features_for(len(dep), channels)
    rng = np.random.default_rng(11)
    grad_f = rng.random((h, w, channels), dtype=np.float32)
    grad_i = rng.random((h, w, 3), dtype=np.float32) if with_rgb else None
    want = oracle.rasterize(*inputs, w, h, background=BACKGROUND, features=feats)
    gm, gc, gcol, go, gf = oracle.render_backward(want["ranges"], want["values"], m2, con, col, opac, w, h,
                                                  want["final_T"], want["n_contrib"], grad_image=grad_i,
                                                  background=BACKGROUND, features=feats, grad_features=grad_f)
    t_in = cuda(*inputs, BACKGROUND)
    f = cuda(feats)[0]
    _, _, final_T, n_contrib, values, ranges, conic, co = ext.rasterize_with_features(*t_in, f, w, h)
    got_m, got_c, got_col, got_o, got_f = ext.rasterize_backward_fused(
        cuda(grad_i)[0] if with_rgb else None, t_in[6], cuda(grad_f)[0], f, t_in[0], conic, co, values, ranges,
        final_T, n_contrib, w, h, half_tile_lists=half_tile_lists)
    from hds_b200.native import device_status

    assert device_status() == 0, "a bounded wait in the feature backward ran out"
    for nm, g, wv in zip(("features", "means2D", "conics", "opacities"), (got_f, got_m, got_c, got_o),
                         (gf, gm, gc, go)):
        assert_grads_close(host(g), wv, nm)
    if with_rgb:
        assert_grads_close(host(got_col), gcol, "colors")
    else:
        assert got_col is None


@pytest.mark.parametrize("channels", [256, 512])
@pytest.mark.parametrize("name", ["raster_ref_scene", "dense_tile", "size3"])
def test_fused_backward_blocks_cut_their_own_lists(ext, golden, monkeypatch, name, channels):
    """Without a workspace every cluster block cuts its half tile's list from the tile list itself;
    the gradients are the oracle's as with the lists cut ahead (256 channels on clusters too)."""
    monkeypatch.setenv("HDS_FEATURE_BWD_CLUSTER", "1")
    test_fused_backward(ext, golden, name, channels, True, half_tile_lists=False)


@pytest.mark.parametrize("name", ["raster_ref_scene", "dense_tile", "size3"])
def test_fused_backward_lists_cut_ahead_256_on_clusters(ext, golden, monkeypatch, name):
    monkeypatch.setenv("HDS_FEATURE_BWD_CLUSTER", "1")
    test_fused_backward(ext, golden, name, 256, True)


def test_fused_backward_workspace_too_small_is_reported(ext, golden):
    """A workspace without room for the frame's pairs: no list is written past it, and the device
    status reports HDS_ERR_TOO_LARGE (the gradients are then incomplete)."""
    import ctypes

    from hds_b200.native import device_status, lib, ptr, stream_of

    inputs, w, h = case("raster_ref_scene", golden)
    feats = features_for(len(inputs[1]), 512)
    t_in = cuda(*inputs, BACKGROUND)
    f = cuda(feats)[0]
    _, _, final_T, n_contrib, values, ranges, conic, co = ext.rasterize_with_features(*t_in, f, w, h)
    n = f.shape[0]
    full = int(lib.hds_backward_workspace_bytes(values.numel(), w, h))
    small = full - 48 * values.numel()  # room for half the slots
    ws = torch.zeros(full, dtype=torch.uint8, device="cuda")
    outs = [torch.zeros(n, k, device="cuda") for k in (3, 512, 2, 3, 1)]
    grad_f = torch.rand(h, w, 512, device="cuda")
    assert device_status() == 0
    rc = lib.hds_render_backward_fused(n, 512, w, h, 0, None, None, ptr(grad_f), ptr(f), ptr(t_in[0]), ptr(conic),
                                       ptr(co), ptr(values), ptr(ranges), ptr(final_T), ptr(n_contrib), None,
                                       *[ptr(t) for t in outs[1:]], 0, ptr(ws), ctypes.c_size_t(small),
                                       stream_of(f.device))
    assert rc == 0
    assert device_status() == 5  # HDS_ERR_TOO_LARGE
    assert device_status() == 0  # read and cleared
    # Nothing was written past the first `small` bytes.
    assert int(ws[small:].count_nonzero()) == 0


def test_unsupported_widths_are_rejected(ext, golden):
    inputs, w, h = case("raster_ref_scene", golden)
    t_in = cuda(*inputs, BACKGROUND)
    _, final_T, n_contrib, values, ranges, conic, co = ext.rasterize(*t_in, w, h)
    with pytest.raises(RuntimeError, match="32, 64, 128, 256 or 512"):
        ext.rasterize_features(torch.rand(len(inputs[1]), 24, device="cuda"), t_in[0], conic, co, values, ranges, w, h)
    f = torch.rand(len(inputs[1]), 256, device="cuda")
    with pytest.raises(RuntimeError, match="no feature backward for 256 channels in slices of 32"):
        ext.rasterize_features_backward(torch.rand(h, w, 256, device="cuda"), f, t_in[0], conic, co, values, ranges,
                                        final_T, n_contrib, w, h, 32)


@pytest.mark.parametrize("which", ["config0", "reference", "config1"])
def test_projection_bit_exact(ext, which):
    from hds_b200 import scenes

    if which == "config0":
        s = scenes.config0(0, channels=0)
        means, sc, q, op, cam = s.means, s.scales, s.quats, s.opacities, s.cameras[0]
    elif which == "config1":
        s = scenes.config1(1, n=50_000, channels=0)
        means, sc, q, op, cam = s.means, s.scales, s.quats, s.opacities, s.cameras[0]
    else:
        g = scenes.reference_test_scene(3, 5000)
        means, sc, q, op = g["means"], g["scales"], g["quats"], g["opacities"]
        cam = scenes.identity_camera(160, 120)
    args = (cam.fx, cam.fy, cam.cx, cam.cy, cam.width, cam.height)
    want = oracle.project_forward(means.numpy(), sc.numpy(), q.numpy(), op.numpy(), cam.world_to_camera.numpy(), *args)
    got = ext.project_gaussians(*cuda(means.numpy(), sc.numpy(), q.numpy(), op.numpy(), cam.world_to_camera.numpy()),
                                *args, oracle.NEAR_PLANE, oracle.LOW_PASS, oracle.FOV_SCALE)
    for nm, g, wv in zip(("means2D", "depths", "radii", "conics"), got, want):
        assert np.array_equal(host(g), wv), f"{nm} differs"
    rng = np.random.default_rng(4)
    gm2 = rng.standard_normal((means.shape[0], 2)).astype(np.float32)
    gcon = rng.standard_normal((means.shape[0], 3)).astype(np.float32)
    want = oracle.project_backward(gm2, gcon, means.numpy(), sc.numpy(), q.numpy(), cam.world_to_camera.numpy(), *args)
    got = ext.project_gaussians_backward(*cuda(gm2, gcon, means.numpy(), sc.numpy(), q.numpy(),
                                               cam.world_to_camera.numpy()), *args, oracle.NEAR_PLANE, oracle.LOW_PASS,
                                         oracle.FOV_SCALE)
    for nm, g, wv in zip(("grad_means", "grad_scales", "grad_quats"), got, want):
        assert np.array_equal(host(g), wv), f"{nm} differs"


def _raw_params(which, zero_quat=True):
    """Raw model parameters whose activations give a test scene: log-scales, quaternions scaled by
    random factors in [0.5, 2) (with zero_quat, one of them zero: the clamp of normalize), opacity
    logits."""
    from hds_b200 import scenes

    s = scenes.config0(0, channels=0) if which == "config0" else scenes.config1(1, n=50_000, channels=0)
    rng = np.random.default_rng(3)
    log_scales = np.log(s.scales.numpy()).astype(np.float32)
    quats = (s.quats.numpy() * rng.uniform(0.5, 2.0, (s.n, 1))).astype(np.float32)
    if zero_quat:
        quats[7] = 0.0
    op = np.clip(s.opacities.numpy(), 1e-6, 1 - 1e-6)
    logits = np.log(op / (1 - op)).astype(np.float32)
    return s.means.numpy(), log_scales, quats, logits, s.cameras[0]


@pytest.mark.parametrize("which", ["config0", "config1"])
def test_projection_raw_bit_exact(ext, which):
    """The projection of raw parameters (exp, normalize and sigmoid in the kernel) equals the oracle's
    activations followed by its projection, forward and backward, bit for bit; the accumulating
    backward adds exactly those gradients."""
    means, ls, q, lg, cam = _raw_params(which)
    args = (cam.fx, cam.fy, cam.cx, cam.cy, cam.width, cam.height)
    consts = (oracle.NEAR_PLANE, oracle.LOW_PASS, oracle.FOV_SCALE)
    sc, unit, op = oracle.activate(ls, q, lg)
    pose = cam.world_to_camera.numpy()
    want = oracle.project_forward(means, sc, unit, op, pose, *args)
    t_means, t_ls, t_q, t_lg, t_pose = cuda(means, ls, q, lg, pose)
    got = ext.project_gaussians_raw(t_means, t_ls, t_q, t_lg, t_pose, *args, *consts)
    for nm, g, wv in zip(("means2D", "depths", "radii", "conics", "opacities"), got, (*want, op)):
        assert np.array_equal(host(g), wv), f"{nm} differs"
    rng = np.random.default_rng(5)
    n = means.shape[0]
    gm2 = rng.standard_normal((n, 2)).astype(np.float32)
    gcon = rng.standard_normal((n, 3)).astype(np.float32)
    gop = rng.standard_normal(lg.shape).astype(np.float32)
    g_means, g_sc, g_unit = oracle.project_backward(gm2, gcon, means, sc, unit, pose, *args)
    g_ls, g_q, g_lg = oracle.activate_backward(ls, q, lg, g_sc, g_unit, gop)
    t_gm2, t_gcon, t_gop = cuda(gm2, gcon, gop)
    got = ext.project_gaussians_raw_backward(t_gm2, t_gcon, t_gop, t_means, t_ls, t_q, t_lg, t_pose, *args, *consts)
    for nm, g, wv in zip(("means", "log_scales", "quats", "logits"), got, (g_means, g_ls, g_q, g_lg)):
        assert np.array_equal(host(g), wv), f"grad {nm} differs"
    bases = [rng.standard_normal(a.shape).astype(np.float32) for a in (means, ls, q, lg)]
    bufs = cuda(*bases)
    ext.project_gaussians_raw_backward(t_gm2, t_gcon, t_gop, t_means, t_ls, t_q, t_lg, t_pose, *args, *consts,
                                       into=bufs)
    for nm, buf, base, wv in zip(("means", "log_scales", "quats", "logits"), bufs, bases,
                                 (g_means, g_ls, g_q, g_lg)):
        assert np.array_equal(host(buf), base + wv), f"accumulated grad {nm} differs"
    got = ext.project_gaussians_raw_backward(t_gm2, t_gcon, None, t_means, t_ls, t_q, t_lg, t_pose, *args, *consts)
    assert np.array_equal(host(got[3]), np.zeros_like(lg)), "no opacity gradient must give zero logit gradients"


@pytest.mark.parametrize("accumulate", [False, True])
def test_projection_raw_matches_torch_activations(ext, accumulate):
    """project_gaussians_raw against the reference's composition (torch exp, normalize and sigmoid,
    then the projection node) through autograd: same outputs within float rounding of the
    activations, and gradients within the gradient tolerance."""
    import torch.nn.functional as F

    from hds_b200.projection import project_gaussians, project_gaussians_raw
    from hds_b200.rasterizer import accumulate_leaf_grads

    # No zero quaternion here: at the clamp both sides divide by 1e-12, and that row would set the
    # gradient tolerance's scale.
    means, ls, q, lg, cam = _raw_params("config1", zero_quat=False)
    args = (cam.fx, cam.fy, cam.cx, cam.cy, cam.width, cam.height)
    pose = cam.world_to_camera.cuda()
    rng = np.random.default_rng(9)
    n = means.shape[0]
    gm2, gcon, gop = (torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).cuda()
                      for shape in ((n, 2), (n, 3), lg.shape))

    def leaves():
        return [torch.from_numpy(a).cuda().requires_grad_(True) for a in (means, ls, q, lg)]

    r = leaves()
    r_out = project_gaussians(r[0], torch.exp(r[1]), F.normalize(r[2], dim=-1), torch.sigmoid(r[3]), pose, *args)
    r_op = torch.sigmoid(r[3])
    torch.autograd.backward([r_out[0], r_out[3], r_op], [gm2, gcon, gop])

    o = leaves()
    if accumulate:
        for t in o:
            t.grad = torch.zeros_like(t)
    with accumulate_leaf_grads() if accumulate else torch.enable_grad():
        o_out = project_gaussians_raw(*o, pose, *args)
    torch.autograd.backward([o_out[0], o_out[3], o_out[4]], [gm2, gcon, gop])
    np.testing.assert_allclose(host(o_out[4]), host(r_op), rtol=1e-6, atol=1e-7)
    vis = (host(o_out[2]) > 0) & (host(r_out[2]) > 0)
    assert vis.mean() > 0.5 and np.mean((host(o_out[2]) > 0) != (host(r_out[2]) > 0)) < 1e-3
    np.testing.assert_allclose(host(o_out[0])[vis], host(r_out[0])[vis], rtol=1e-5, atol=1e-3)
    for nm, a, b in zip(("means", "log_scales", "quats", "logits"), o, r):
        assert_grads_close(host(a.grad), host(b.grad), nm)


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
def test_sh_bit_exact(ext, golden, degree):
    g = golden("sh.npz")
    sh, dirs, radii, grad_rgb = g["sh"], g["dirs"], g["radii"], g["grad_rgb"]
    dc, rest = np.ascontiguousarray(sh[:, :1]), np.ascontiguousarray(sh[:, 1:])
    t_dc, t_rest, t_dirs, t_radii, t_grad = cuda(dc, rest, dirs, radii, grad_rgb)
    assert np.array_equal(host(ext.eval_sh(t_dc, t_rest, t_dirs, degree, t_radii)),
                          oracle.eval_sh(dc, rest, dirs, degree, radii))
    got = ext.eval_sh_backward(t_grad, t_dc, t_rest, t_dirs, degree, t_radii)
    want = oracle.eval_sh_backward(grad_rgb, dc, rest, dirs, degree, radii)
    for nm, a, b in zip(("dc", "rest", "dirs"), got, want):
        assert np.array_equal(host(a), b), f"grad {nm} differs"


def test_sh_adam_matches_oracle_and_torch(ext, golden):
    g = golden("sh.npz")
    sh, dirs, radii = g["sh"], g["dirs"], g["radii"]
    dc, rest = np.ascontiguousarray(sh[:, :1]), np.ascontiguousarray(sh[:, 1:])
    t_dc, t_rest, t_dirs, t_radii = cuda(dc, rest, dirs, radii)
    m_dc, v_dc, m_rest, v_rest = (torch.zeros_like(t) for t in (t_dc, t_dc, t_rest, t_rest))
    step = torch.zeros((), device="cuda")
    o_state = {"dc": (np.zeros_like(dc), np.zeros_like(dc)), "rest": (np.zeros_like(rest), np.zeros_like(rest))}
    for k, grad_rgb in enumerate(g["adam_grad_rgb"], start=1):
        step += 1
        ext.eval_sh_backward_adam(cuda(grad_rgb)[0], t_dc, t_rest, t_dirs, 3, t_radii, m_dc, v_dc, m_rest, v_rest, step,
                                  step, 0.0025, 0.0025 / 20, 0.9, 0.999, 1e-15)
        gdc, grest, _ = oracle.eval_sh_backward(grad_rgb, dc, rest, dirs, 3, radii)
        dc, m, v = oracle.adam(dc, *o_state["dc"], gdc, k, 0.0025, 0.9, 0.999, 1e-15)
        o_state["dc"] = (m, v)
        rest, m, v = oracle.adam(rest, *o_state["rest"], grest, k, 0.0025 / 20, 0.9, 0.999, 1e-15)
        o_state["rest"] = (m, v)
    np.testing.assert_allclose(host(t_dc), dc, rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(host(t_rest), rest, rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(host(t_dc), g["adam_dc"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(host(t_rest), g["adam_rest"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(host(m_rest), g["adam_m_rest"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(host(v_rest), g["adam_v_rest"], rtol=1e-5, atol=1e-7)


def _sh_inputs(n, seed):
    rng = np.random.default_rng(seed)
    sh = (0.5 * rng.standard_normal((n, 16, 3))).astype(np.float32)
    d = rng.standard_normal((n, 3))
    dirs = (d / np.linalg.norm(d, axis=1, keepdims=True)).astype(np.float32)
    radii = rng.integers(0, 3, n).astype(np.float32)  # about a third culled
    grad_rgb = rng.standard_normal((n, 3)).astype(np.float32)
    return np.ascontiguousarray(sh[:, :1]), np.ascontiguousarray(sh[:, 1:]), dirs, radii, grad_rgb


def _placed(a, offset):
    """A CUDA copy of `a` that starts `offset` floats into a larger buffer (offset 1 breaks 16-byte
    alignment and sends the SH kernels down their element-by-element path)."""
    flat = torch.zeros(a.size + offset, dtype=torch.float32, device="cuda")
    flat[offset:] = torch.from_numpy(np.ascontiguousarray(a).reshape(-1)).cuda()
    return flat[offset:].view(a.shape)


@pytest.mark.parametrize("n,offset", [(1000, 0), (1000, 1), (128, 0), (37, 0)])
@pytest.mark.parametrize("degree", [0, 3])
def test_sh_blocks_and_alignment(ext, n, offset, degree):
    """Whole 128-gaussian blocks (vector loads), a partial last block and unaligned inputs (element
    loads) give the oracle's colours and gradients bit for bit; the accumulating backward adds
    exactly the plain gradient to what its buffers hold."""
    dc, rest, dirs, radii, grad_rgb = _sh_inputs(n, 7 * n + offset)
    t_dc, t_rest = _placed(dc, offset), _placed(rest, offset)
    t_dirs, t_radii, t_grad = cuda(dirs, radii, grad_rgb)
    assert np.array_equal(host(ext.eval_sh(t_dc, t_rest, t_dirs, degree, t_radii)),
                          oracle.eval_sh(dc, rest, dirs, degree, radii))
    want = oracle.eval_sh_backward(grad_rgb, dc, rest, dirs, degree, radii)
    got = ext.eval_sh_backward(t_grad, t_dc, t_rest, t_dirs, degree, t_radii)
    for nm, a, b in zip(("dc", "rest", "dirs"), got, want):
        assert np.array_equal(host(a), b), f"grad {nm} differs"
    rng = np.random.default_rng(n)
    base_dc = rng.standard_normal(dc.shape).astype(np.float32)
    base_rest = rng.standard_normal(rest.shape).astype(np.float32)
    buf_dc, buf_rest = _placed(base_dc, offset), _placed(base_rest, offset)
    gd = ext.eval_sh_backward_into(buf_dc, buf_rest, t_grad, t_dc, t_rest, t_dirs, degree, t_radii)
    assert np.array_equal(host(buf_dc), base_dc + want[0])
    assert np.array_equal(host(buf_rest), base_rest + want[1])
    assert np.array_equal(host(gd), want[2])


@pytest.mark.parametrize("n,offset", [(1000, 0), (1000, 1)])
def test_sh_adam_blocks_and_alignment(ext, n, offset):
    """The fused Adam step on whole blocks (float4 parameter and moment traffic), a partial block and
    unaligned buffers, against the oracle's gradient and Adam."""
    dc, rest, dirs, radii, _ = _sh_inputs(n, 11 * n + offset)
    t_dc, t_rest = _placed(dc, offset), _placed(rest, offset)
    t_dirs, t_radii = cuda(dirs, radii)
    m_dc, v_dc = _placed(np.zeros_like(dc), offset), _placed(np.zeros_like(dc), offset)
    m_rest, v_rest = _placed(np.zeros_like(rest), offset), _placed(np.zeros_like(rest), offset)
    step = torch.zeros((), device="cuda")
    o_dc, o_rest = (np.zeros_like(dc), np.zeros_like(dc)), (np.zeros_like(rest), np.zeros_like(rest))
    rng = np.random.default_rng(n + offset)
    for k in range(1, 4):
        grad_rgb = rng.standard_normal((n, 3)).astype(np.float32)
        step += 1
        ext.eval_sh_backward_adam(cuda(grad_rgb)[0], t_dc, t_rest, t_dirs, 3, t_radii, m_dc, v_dc, m_rest, v_rest,
                                  step, step, 0.0025, 0.0025 / 20, 0.9, 0.999, 1e-15)
        gdc, grest, _ = oracle.eval_sh_backward(grad_rgb, dc, rest, dirs, 3, radii)
        dc, *o_dc = oracle.adam(dc, *o_dc, gdc, k, 0.0025, 0.9, 0.999, 1e-15)
        rest, *o_rest = oracle.adam(rest, *o_rest, grest, k, 0.0025 / 20, 0.9, 0.999, 1e-15)
    np.testing.assert_allclose(host(t_dc), dc, rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(host(t_rest), rest, rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(host(m_rest), o_rest[0], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(host(v_rest), o_rest[1], rtol=1e-6, atol=1e-7)


def _view_inputs(n, seed):
    dc, rest, _, radii, grad_rgb = _sh_inputs(n, seed)
    rng = np.random.default_rng(seed + 1)
    center = rng.standard_normal(3).astype(np.float32)
    means = (center + 5.0 * rng.standard_normal((n, 3))).astype(np.float32)
    means[3] = center  # |means - center| = 0: the 1e-12 clamp of normalize
    radii[3] = 1.0
    return dc, rest, means, center, radii, grad_rgb


@pytest.mark.parametrize("n", [1000, 128, 37])
@pytest.mark.parametrize("degree", [0, 3])
def test_sh_view_bit_exact(ext, n, degree):
    """eval_sh_view forms normalize(means - camera_center) in the kernel: colours, SH gradients and
    dL/dmeans equal the oracle's float32 restatement bit for bit, including a mean at the centre."""
    dc, rest, means, center, radii, grad_rgb = _view_inputs(n, 5 * n + degree)
    dirs, s = oracle.view_dirs(means, center)
    t_dc, t_rest, t_means, t_center, t_radii, t_grad = cuda(dc, rest, means, center, radii, grad_rgb)
    assert np.array_equal(host(ext.eval_sh_view(t_dc, t_rest, t_means, t_center, degree, t_radii)),
                          oracle.eval_sh(dc, rest, dirs, degree, radii))
    gdc, grest, gdirs = oracle.eval_sh_backward(grad_rgb, dc, rest, dirs, degree, radii)
    gmeans = oracle.view_dirs_backward(gdirs, dirs, s)
    got = ext.eval_sh_view_backward(t_grad, t_dc, t_rest, t_means, t_center, degree, t_radii)
    for nm, a, b in zip(("dc", "rest", "means"), got, (gdc, grest, gmeans)):
        assert np.array_equal(host(a), b), f"grad {nm} differs"
    rng = np.random.default_rng(n)
    bases = [rng.standard_normal(a.shape).astype(np.float32) for a in (dc, rest, means)]
    bufs = cuda(*bases)
    ext.eval_sh_view_backward(t_grad, t_dc, t_rest, t_means, t_center, degree, t_radii, into=bufs)
    for nm, buf, base, g in zip(("dc", "rest", "means"), bufs, bases, (gdc, grest, gmeans)):
        assert np.array_equal(host(buf), base + g), f"accumulated grad {nm} differs"


@pytest.mark.parametrize("accumulate", [False, True])
def test_view_colors_matches_torch_normalize(ext, accumulate):
    """view_colors against the reference's composition, F.normalize(means - camera_center) followed by
    the SH node, through autograd: same colours, and gradients within the gradient tolerance (torch's
    normalize backward rounds differently).  With accumulate_leaf_grads the gradients land in the
    leaves' existing .grad buffers; a camera centre that needs a gradient gets -sum dL/dmeans."""
    import torch.nn.functional as F

    from hds_b200.rasterizer import accumulate_leaf_grads
    from hds_b200.sh import eval_sh_grad, view_colors

    dc, rest, means, center, radii, grad_rgb = _view_inputs(3000, 17)
    means[3] += 1.0  # keep the reference composition away from its clamp, where torch's gradient is 0 * inf
    t_radii, t_grad = cuda(radii, grad_rgb)

    def leaves(center_grad):
        out = [torch.from_numpy(a).cuda().requires_grad_(True) for a in (dc, rest, means)]
        return out + [torch.from_numpy(center).cuda().requires_grad_(center_grad)]

    r_dc, r_rest, r_means, r_center = leaves(True)
    ref = eval_sh_grad(r_dc, r_rest, F.normalize(r_means - r_center, dim=-1), 3, t_radii)
    ref.backward(t_grad)

    o_dc, o_rest, o_means, o_center = leaves(not accumulate)
    if accumulate:
        for t in (o_dc, o_rest, o_means):
            t.grad = torch.zeros_like(t)
    with accumulate_leaf_grads() if accumulate else torch.enable_grad():
        rgb = view_colors(o_dc, o_rest, o_means, o_center, 3, t_radii)
    rgb.backward(t_grad)
    np.testing.assert_allclose(host(rgb), host(ref), rtol=0, atol=1e-5)
    for nm, a, b in (("sh_dc", o_dc, r_dc), ("sh_rest", o_rest, r_rest), ("means", o_means, r_means)):
        assert_grads_close(host(a.grad), host(b.grad), nm)
    if not accumulate:
        assert_grads_close(host(o_center.grad), host(r_center.grad), "camera_center")


def test_sh_grad_accumulates_into_leaf_grads(ext):
    """eval_sh_grad under accumulate_leaf_grads adds its SH gradients into existing leaf .grad buffers
    (and returns the same dL/ddirs); without buffers it falls back to autograd's own accumulation."""
    from hds_b200.rasterizer import accumulate_leaf_grads
    from hds_b200.sh import eval_sh_grad

    dc, rest, dirs, radii, grad_rgb = _sh_inputs(700, 3)
    want = oracle.eval_sh_backward(grad_rgb, dc, rest, dirs, 3, radii)
    for preset in (True, False):
        t_dc, t_rest = (torch.from_numpy(a).cuda().requires_grad_(True) for a in (dc, rest))
        t_dirs = torch.from_numpy(dirs).cuda().requires_grad_(True)
        t_radii, t_grad = cuda(radii, grad_rgb)
        if preset:
            t_dc.grad, t_rest.grad = torch.ones_like(t_dc), torch.ones_like(t_rest)
        with accumulate_leaf_grads():
            rgb = eval_sh_grad(t_dc, t_rest, t_dirs, 3, t_radii)
        rgb.backward(t_grad)
        base = 1.0 if preset else 0.0
        assert np.array_equal(host(t_dc.grad), want[0] + np.float32(base))
        assert np.array_equal(host(t_rest.grad), want[1] + np.float32(base))
        assert np.array_equal(host(t_dirs.grad), want[2])


@pytest.mark.parametrize("size", ["64x64", "37x53", "11x11", "546x979"])
def test_ssim_bit_exact(ext, golden, size):
    if size == "546x979":
        rng = np.random.default_rng(0)
        b = rng.random((546, 979, 3), dtype=np.float32)
        a = np.clip(b + 0.1 * rng.standard_normal(b.shape).astype(np.float32), 0, 1).astype(np.float32)
    else:
        g = golden("ssim.npz")
        a, b = g[f"{size}_rendered"], g[f"{size}_gt"]
    want = oracle.ssim_forward(a, b)
    ta, tb = cuda(a, b)
    got = ext.ssim_forward(ta, tb)
    for nm, x, y in zip(("map", "d_mu", "d_aa", "d_ab"), got, want):
        assert np.array_equal(host(x), y), f"ssim {nm} differs"
    grad_mean = torch.full((1,), 0.37, device="cuda")
    got = ext.ssim_backward(grad_mean, ta, tb, *got[1:])
    assert np.array_equal(host(got), oracle.ssim_backward(np.float32(0.37), a, b, *want[1:]))
    if size != "546x979":
        np.testing.assert_allclose(host(ext.ssim_forward(ta, tb)[0]).astype(np.float64).mean(),
                                   golden("ssim.npz")[f"{size}_ssim"], rtol=1e-5, atol=1e-6)


def test_no_device_side_failures(ext):
    from hds_b200.native import device_status

    assert device_status() == 0

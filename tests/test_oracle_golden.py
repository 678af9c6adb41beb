"""Pins the C oracle (oracle/hds_oracle.c) to the reference before anything is compared with it.

* The golden fixtures hold outputs of the reference's own fp64 oracle, SH reference and torch SSIM
  (tests/golden/make_golden.py).  FP32 with a fixed order against fp64: images within 1e-5,
  gradients within 1e-4 of the largest gradient (a pair that lands exactly on the MIN_ALPHA or
  MIN_T cutoff may flip between the two precisions, so 0.1% of entries may be further off).
* The hand-solved single-pixel cases are those of the reference's tests/test_oracle.py:28-44.
* The edge-case assertions are those of the reference's tests/test_render.py:183-225.
"""
import math

import numpy as np
import pytest

import oracle
from helpers import RGB_ATOL, assert_close_abs, assert_grads_close, seeded_uniform

BACKGROUND = (0.3, 0.5, 0.7)


def render_one_pixel(opacities):
    """Gaussians stacked on the centre of a 1x1 image, front to back, gaussian i coloured with channel i."""
    n = len(opacities)
    out = oracle.rasterize(np.full((n, 2), 0.5), np.arange(n), np.ones(n), np.tile([1.0, 0.0, 1.0], (n, 1)),
                           np.eye(3)[:n].reshape(n, 3), np.asarray(opacities).reshape(n, 1), 1, 1,
                           background=np.asarray(BACKGROUND))
    return out["image"][0, 0]


@pytest.mark.parametrize("opacities, expected", [
    ([0.5], [0.5 + 0.5 * 0.3, 0.5 * 0.5, 0.5 * 0.7]),
    # The reference's fp64 oracle expects [0.99 + 1e-4*0.3, 0.0099 + 1e-4*0.5, 1e-4*0.7]: its
    # second gaussian leaves T = 0.01 * 0.01, exactly the 1e-4 floor.  In FP32 (the reference's
    # forward.cu:212-216 and this oracle alike) 1 - 0.99f = 0.0099999905 and the product rounds to
    # 9.99998e-5 < 1e-4f, so the walk stops before the second gaussian.
    ([1.0, 1.0, 1.0], [0.99 + 0.01 * 0.3, 0.01 * 0.5, 0.01 * 0.7]),
    ([0.99, 0.5, 0.99], [0.99 + 0.005 * 0.3, 0.005 + 0.005 * 0.5, 0.005 * 0.7]),
    ([], list(BACKGROUND)),
])
def test_hand_solved_pixel(opacities, expected):
    np.testing.assert_allclose(render_one_pixel(opacities), expected, atol=1e-6)


def test_expf_logf_accuracy():
    xs = np.linspace(-87.0, 10.0, 20011, dtype=np.float32)
    rel = max(abs(oracle.expf(x) - math.exp(float(x))) / math.exp(float(x)) for x in xs)
    assert rel < 1.2e-7
    ys = np.exp(np.linspace(-20, 20, 20011)).astype(np.float32)
    err = max(abs(oracle.logf(y) - math.log(float(y))) / max(1.0, abs(math.log(float(y)))) for y in ys)
    assert err < 2.5e-7


def test_ssim_window_matches_reference(golden):
    # The reference's torch path blurs with the [11, 11] outer product of the 1-D window
    # (loss.py:35-38); ssim.cu:12-15 hardcodes the 1-D taps.
    g = golden("ssim.npz")
    w = oracle.ssim_window().astype(np.float64)
    np.testing.assert_allclose(np.outer(w, w), g["window"], rtol=1e-6, atol=0)


def check_raster(fix, rgb_bad_fraction=0.0):
    w, h = int(fix["width"]), int(fix["height"])
    inputs = [fix[k] for k in ("means2D", "depths", "radii", "conics", "colors", "opacities")]
    m2, dep, rad, con, col, opac = inputs
    r = oracle.rasterize(*inputs, w, h, background=fix["background"], features=fix["features"])
    assert_close_abs(r["image"], fix["image"], RGB_ATOL, "image")
    assert_close_abs(r["features"], fix["feature_image"], 1e-5, "feature image")
    # The split-bf16 contraction the tensor cores compute (hi*hi + hi*lo + lo*hi of each weight and
    # feature) stays inside the 1e-3 absolute feature tolerance whatever the features' magnitude
    # (config 0 draws them N(0, 1)); plain TF32 rounding of both factors would not (1.6e-3 there).
    rs = oracle.render_forward(r["ranges"], r["values"], m2, con, None, opac, w, h, features=fix["features"],
                               split_bf16=True)[3]
    assert_close_abs(rs, fix["feature_image"], 1e-3, "split-bf16 feature image")
    gi = fix["grad_image"] if "grad_image" in fix else seeded_uniform(int(fix["grad_image_seed"]), (h, w, 3))
    gf = fix["grad_features"] if "grad_features" in fix else seeded_uniform(int(fix["grad_features_seed"]),
                                                                             (h, w, fix["features"].shape[1]))
    gm, gc, gcol, go, _ = oracle.render_backward(r["ranges"], r["values"], m2, con, col, opac, w, h, r["final_T"],
                                                 r["n_contrib"], grad_image=gi, background=fix["background"])
    for name, got in (("means2D", gm), ("conics", gc), ("colors", gcol), ("opacities", go)):
        assert_grads_close(got, fix[f"grad_{name}"], name)
    gm, gc, _, go, gfeat = oracle.render_backward(r["ranges"], r["values"], m2, con, None, opac, w, h, r["final_T"],
                                                  r["n_contrib"], features=fix["features"], grad_features=gf)
    for name, got in (("means2D", gm), ("conics", gc), ("features", gfeat), ("opacities", go)):
        assert_grads_close(got, fix[f"feat_grad_{name}"], "feature " + name)
    return r


def test_reference_scene_matches_golden(golden):
    check_raster(golden("raster_ref_scene.npz"))


def test_config0_matches_golden(golden):
    r = check_raster(golden("raster_config0.npz"))
    assert len(r["keys"]) > 4096, "config 0 should produce duplicates across tiles"


@pytest.mark.parametrize("case", ["depth_ties", "min_alpha", "max_alpha", "t_floor", "dense_tile"])
def test_flat_edge_cases_match_golden(golden, case):
    g = golden("raster_flat.npz")
    fix = {k.split("__", 1)[1]: v for k, v in g.items() if k.startswith(case + "__")}
    fix["width"], fix["height"] = fix["size"]
    fix["background"] = g["background"]
    check_raster(fix)


def test_flat_edge_case_assertions():
    def flat(means, depths, sigmas, opacities):
        k = len(depths)
        s = np.asarray(sigmas, np.float32)
        cols = np.random.default_rng(k).random((k, 3), dtype=np.float32)
        return (np.asarray(means, np.float32), np.asarray(depths, np.float32), np.ones(k, np.float32),
                np.stack([s ** -2, 0 * s, s ** -2], -1), cols, np.asarray(opacities, np.float32)[:, None])

    # test_render.py:183-188: equal depths blend in index order, so swapping them changes the image.
    ties = flat([[7.5, 8.5], [9.5, 8.5]], [2.0, 2.0], [3.0, 3.0], [0.7, 0.7])
    swapped = tuple(x[::-1].copy() for x in ties)
    assert not np.array_equal(oracle.rasterize(*ties, 16, 16)["image"], oracle.rasterize(*swapped, 16, 16)["image"])
    # test_render.py:191-197: just above MIN_ALPHA blends, just below does not.
    ma = flat([[4.5, 4.5], [12.5, 4.5]], [1.0, 1.0], [0.5, 0.5], [1.01 / 255, 0.99 / 255])
    img = oracle.rasterize(*ma, 16, 8)["image"]
    assert np.abs(img[4, 4]).sum() > 0 and np.array_equal(img[4, 12], np.zeros(3, np.float32))
    # test_render.py:200-205: opacity 1 clamps to 0.99.
    mx = flat([[8.5, 8.5]], [1.0], [2.0], [1.0])
    np.testing.assert_allclose(oracle.rasterize(*mx, 16, 16)["image"][8, 8], 0.99 * mx[4][0], rtol=1e-6)
    # test_render.py:214-225: a dense tile walks past the 256-entry batch edge.
    r = np.random.default_rng(11)
    dense = flat((r.random((2000, 2)) * 16).tolist(), (1 + r.random(2000)).tolist(), [12.0] * 2000, [0.02] * 2000)
    assert oracle.rasterize(*dense, 16, 16)["n_contrib"].min() > 256


def test_binning_is_sorted_and_ranges_cover_keys(golden):
    fix = golden("raster_config0.npz")
    w, h = int(fix["width"]), int(fix["height"])
    touched, keys, values, ranges = oracle.bin_gaussians(fix["means2D"], fix["depths"], fix["radii"], fix["conics"],
                                                         fix["opacities"], w, h)
    assert len(keys) == touched.sum()
    assert np.all(keys[1:] >= keys[:-1])
    tiles = (keys >> np.uint64(32)).astype(np.int64)
    for t in np.unique(tiles):
        idx = np.nonzero(tiles == t)[0]
        assert ranges[t, 0] == idx[0] and ranges[t, 1] == idx[-1] + 1
    depth_bits = (keys & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    assert np.array_equal(depth_bits, fix["depths"][values].view(np.uint32))
    # Stable: equal keys keep gaussian index order.
    same = keys[1:] == keys[:-1]
    assert np.all(values[1:][same] > values[:-1][same])


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
def test_sh_matches_golden(golden, degree):
    g = golden("sh.npz")
    sh, dirs, radii = g["sh"], g["dirs"], g["radii"]
    rgb = oracle.eval_sh(sh[:, :1], sh[:, 1:], dirs, degree, radii)
    np.testing.assert_allclose(rgb, g[f"rgb_{degree}"], rtol=1e-5, atol=1e-6)
    gdc, grest, gd = oracle.eval_sh_backward(g["grad_rgb"], sh[:, :1], sh[:, 1:], dirs, degree, radii)
    np.testing.assert_allclose(np.concatenate([gdc, grest], 1), g[f"grad_sh_{degree}"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(gd, g[f"grad_dirs_{degree}"], rtol=1e-4, atol=1e-5)


def test_sh_adam_matches_torch_adam(golden):
    g = golden("sh.npz")
    sh, dirs, radii = g["sh"], g["dirs"], g["radii"]
    dc, rest = sh[:, :1].copy(), sh[:, 1:].copy()
    state = {k: (np.zeros_like(p), np.zeros_like(p)) for k, p in (("dc", dc), ("rest", rest))}
    for step, grad_rgb in enumerate(g["adam_grad_rgb"], start=1):
        gdc, grest, _ = oracle.eval_sh_backward(grad_rgb, dc, rest, dirs, 3, radii)
        dc, m, v = oracle.adam(dc, *state["dc"], gdc, step, 0.0025, 0.9, 0.999, 1e-15)
        state["dc"] = (m, v)
        rest, m, v = oracle.adam(rest, *state["rest"], grest, step, 0.0025 / 20, 0.9, 0.999, 1e-15)
        state["rest"] = (m, v)
    np.testing.assert_allclose(dc, g["adam_dc"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(rest, g["adam_rest"], rtol=1e-5, atol=1e-6)
    for key in ("dc", "rest"):
        np.testing.assert_allclose(state[key][0], g[f"adam_m_{key}"], rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(state[key][1], g[f"adam_v_{key}"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("size", ["64x64", "37x53", "11x11"])
def test_ssim_matches_golden(golden, size):
    g = golden("ssim.npz")
    a, b = g[f"{size}_rendered"], g[f"{size}_gt"]
    smap, d_mu, d_aa, d_ab = oracle.ssim_forward(a, b)
    np.testing.assert_allclose(smap.astype(np.float64).mean(), g[f"{size}_ssim"], rtol=1e-5, atol=1e-6)
    grad = oracle.ssim_backward(1.0, a, b, d_mu, d_aa, d_ab)
    np.testing.assert_allclose(grad, g[f"{size}_grad"], rtol=1e-3, atol=1e-9)
    s_self = oracle.ssim_forward(b, b)[0]
    np.testing.assert_allclose(s_self.astype(np.float64).mean(), 1.0, atol=1e-6)

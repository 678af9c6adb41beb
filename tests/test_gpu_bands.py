"""Bands of rows (origin_y) through the C ABI: a band rendered as an image of its own, with the means
in full-image pixels, equals those rows of the full render bit for bit -- RGB, final T, contributor
counts and the 512- and 32-channel feature images -- and matches the oracle's band render; band
backward passes sum to the full image's gradients."""
import numpy as np
import pytest

import oracle
from hds_b200 import parallel
from helpers import assert_grads_close
from scenes_np import config_scene

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

BACKGROUND = np.array([0.3, 0.5, 0.7], np.float32)


@pytest.fixture(scope="module")
def scene():
    from hds_b200 import scenes

    inputs, cam = config_scene(scenes.config1(2, n=20_000, channels=0))
    return inputs, cam.width, cam.height


def cuda(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]


def host(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("channels", [32, 512])
@pytest.mark.parametrize("world", [2, 5])
def test_band_forward_equals_full_rows(scene, channels, world):
    from hds_b200 import gaussian_rasterizer as ext

    inputs, w, h = scene
    feats = np.random.default_rng(channels).standard_normal((len(inputs[1]), channels)).astype(np.float32)
    t_in = cuda(*inputs, BACKGROUND)
    f = cuda(feats)[0]
    full = ext.rasterize_with_features(*t_in, f, w, h)
    for y0, y1 in parallel.row_bands(h, world):
        band = ext.rasterize_with_features(*t_in, f, w, y1 - y0, origin_y=y0)
        for name, a, b in zip(("image", "features", "final_T", "n_contrib"), band[:4], full[:4]):
            assert torch.equal(a, b[y0:y1]), f"band [{y0}, {y1}) {name} differs from the full render's rows"
        want = oracle.rasterize(*inputs, w, y1 - y0, background=BACKGROUND, origin_y=y0)
        assert np.array_equal(host(band[0]), want["image"]) and np.array_equal(host(band[3]), want["n_contrib"])


def test_band_backward_sums_to_full(scene):
    from hds_b200 import gaussian_rasterizer as ext

    inputs, w, h = scene
    m2, dep, rad, con, col, opac = inputs
    C = 512
    feats = np.random.default_rng(5).standard_normal((len(dep), C)).astype(np.float32)
    rng = np.random.default_rng(6)
    grad_f = rng.random((h, w, C), dtype=np.float32)
    grad_i = rng.random((h, w, 3), dtype=np.float32)
    t_in = cuda(*inputs, BACKGROUND)
    f = cuda(feats)[0]
    full = oracle.rasterize(*inputs, w, h, background=BACKGROUND)
    want = oracle.render_backward(full["ranges"], full["values"], m2, con, col, opac, w, h, full["final_T"],
                                  full["n_contrib"], grad_image=grad_i, background=BACKGROUND, features=feats,
                                  grad_features=grad_f)
    sums = None
    for y0, y1 in parallel.row_bands(h, 3):
        out = ext.rasterize_with_features(*t_in, f, w, y1 - y0, origin_y=y0)
        _, _, final_T, n_contrib, values, ranges, conic, co = out
        got = ext.rasterize_backward_fused(cuda(grad_i[y0:y1])[0], t_in[6], cuda(grad_f[y0:y1])[0], f, t_in[0], conic,
                                           co, values, ranges, final_T, n_contrib, w, y1 - y0, origin_y=y0)
        band = oracle.render_backward(host(ranges), host(values), m2, con, col, opac, w, y1 - y0, host(final_T),
                                      host(n_contrib), grad_image=grad_i[y0:y1], background=BACKGROUND,
                                      features=feats, grad_features=grad_f[y0:y1], origin_y=y0)
        for nm, g, wv in zip(("means2D", "conics", "colors", "opacities", "features"), got, band):
            assert_grads_close(host(g), wv, f"band [{y0}, {y1}) {nm}")
        parts = [host(g).astype(np.float64) for g in got]
        sums = parts if sums is None else [a + b for a, b in zip(sums, parts)]
    for nm, g, wv in zip(("means2D", "conics", "colors", "opacities", "features"), sums, want):
        assert_grads_close(g, wv, f"sum of bands {nm}")

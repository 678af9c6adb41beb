"""Test scenes as numpy 2-D rasterizer inputs (means2D, depths, radii, conics, colors, opacities).

Projected scenes use the oracle's projection; flat scenes and the reference-scene / config-0 inputs
come from the golden fixtures.
"""
from __future__ import annotations

import numpy as np

import oracle
from hds_b200 import scenes

GOLDEN_FLAT_CASES = ["depth_ties", "min_alpha", "max_alpha", "t_floor", "dense_tile"]

# The reference's tests/scenes.py:74-80 size examples, as (seed, n, width, height).
SIZE_EXAMPLES = [(0, 0, 1, 1), (1, 1, 1, 1), (2, 3000, 16, 16), (3, 3000, 17, 17), (4, 10_000, 16, 16)]


def project_np(means, scales, quats, opacities, cam):
    return oracle.project_forward(means, scales, quats, opacities, cam.world_to_camera.numpy(), cam.fx, cam.fy, cam.cx,
                                  cam.cy, cam.width, cam.height)


def reference_scene(seed: int, n: int, width: int, height: int, channels: int = 3):
    """The reference tests' scene (tests/scenes.py:15-54): projected through the identity camera."""
    g = scenes.reference_test_scene(seed, n, channels)
    cam = scenes.identity_camera(width, height)
    m2, dep, rad, con = project_np(g["means"].numpy(), g["scales"].numpy(), g["quats"].numpy(),
                                   g["opacities"].numpy(), cam)
    return m2, dep, rad, con, g["colors"].numpy(), g["opacities"].numpy()


def config_scene(s: scenes.Scene, view: int = 0):
    cam = s.cameras[view]
    m2, dep, rad, con = project_np(s.means.numpy(), s.scales.numpy(), s.quats.numpy(), s.opacities.numpy(), cam)
    colors = np.random.default_rng(7).random((s.n, 3), dtype=np.float32)
    return (m2, dep, rad, con, colors, s.opacities.numpy()), cam


def golden_case(golden, name):
    if name in ("raster_ref_scene", "raster_config0"):
        fix = golden(name + ".npz")
    else:
        g = golden("raster_flat.npz")
        fix = {k.split("__", 1)[1]: v for k, v in g.items() if k.startswith(name + "__")}
        fix["width"], fix["height"] = fix["size"]
        fix["background"] = g["background"]
    inputs = tuple(fix[k] for k in ("means2D", "depths", "radii", "conics", "colors", "opacities"))
    return inputs, int(fix["width"]), int(fix["height"]), fix

"""numpy front end of the C oracle (oracle/hds_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the cpu_baseline
leg of bench.py, never by the product.  Each wrapper names the reference function it restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
SOURCE = HERE / "hds_oracle.c"

TILE = 16
MIN_ALPHA = np.float32(1.0) / np.float32(255.0)
MAX_ALPHA = np.float32(0.99)
MIN_T = np.float32(1e-4)
NEAR_PLANE, LOW_PASS, FOV_SCALE = 0.2, 0.3, 1.3


def build(force: bool = False) -> Path:
    """Compiles hds_oracle.c into liboracle.so beside it (gcc, no FMA contraction)."""
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < SOURCE.stat().st_mtime:
        tmp = LIB_PATH.with_suffix(f".{os.getpid()}.tmp")
        subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
                        str(SOURCE), "-o", str(tmp), "-lm"], check=True)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


_lib = None
F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
F64P = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
U64P = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
c_int, c_float, c_i64 = ctypes.c_int, ctypes.c_float, ctypes.c_int64
vp = ctypes.c_void_p


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        L = _lib
        L.oracle_expf.restype = c_float
        L.oracle_expf.argtypes = [c_float]
        L.oracle_logf.restype = c_float
        L.oracle_logf.argtypes = [c_float]
        L.oracle_tf32_rna.restype = c_float
        L.oracle_tf32_rna.argtypes = [c_float]
        L.oracle_bf16_rne.restype = c_float
        L.oracle_bf16_rne.argtypes = [c_float]
        L.oracle_ssim_window.argtypes = [F32P]
        L.oracle_project_forward.argtypes = [c_int, F32P, F32P, F32P, F32P, F32P, c_float, c_float, c_float, c_float,
                                             c_int, c_int, c_float, c_float, c_float, F32P, F32P, F32P, F32P]
        L.oracle_project_backward.argtypes = [c_int, F32P, F32P, F32P, F32P, F32P, F32P, c_float, c_float, c_float,
                                              c_float, c_int, c_int, c_float, c_float, c_float, F32P, F32P, F32P]
        L.oracle_activate.argtypes = [c_int, F32P, F32P, F32P, F32P, F32P, F32P]
        L.oracle_activate_backward.argtypes = [c_int, F32P, F32P, F32P, F32P, F32P, vp, F32P, F32P, F32P]
        L.oracle_eval_sh_forward.argtypes = [c_int, c_int, F32P, F32P, F32P, F32P, F32P]
        L.oracle_eval_sh_backward.argtypes = [c_int, c_int, F32P, F32P, F32P, F32P, F32P, F32P, F32P, F32P]
        L.oracle_adam.argtypes = [c_int, F32P, F32P, F32P, F32P, c_float, c_float, c_float, c_float, c_float,
                                  c_float, c_float]
        L.oracle_bin.restype = c_i64
        L.oracle_bin.argtypes = [c_int, F32P, F32P, F32P, F32P, F32P, c_int, c_int, c_int, c_i64, vp, vp, vp, vp]
        L.oracle_render_forward.argtypes = [c_int, c_int, c_int, I32P, I32P, F32P, F32P, vp, F32P, vp, c_int, vp,
                                            c_int, vp, vp, vp, vp]
        L.oracle_render_backward.argtypes = [c_int, c_int, c_int, I32P, I32P, F32P, F32P, vp, F32P, vp, F32P, I32P,
                                             vp, c_int, vp, vp, F64P, F64P, F64P, F64P, vp]
        L.oracle_ssim_forward.argtypes = [c_int, c_int, F32P, F32P, F32P, F32P, F32P, F32P]
        L.oracle_ssim_backward.argtypes = [c_int, c_int, c_float, F32P, F32P, F32P, F32P, F32P, F32P]
    return _lib


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def expf(x: float) -> float:
    return lib().oracle_expf(float(x))


def logf(x: float) -> float:
    return lib().oracle_logf(float(x))


def bf16(x: np.ndarray) -> np.ndarray:
    """__float2bfloat16_rn applied elementwise (returned as float32)."""
    u = f32(x).view(np.uint32).copy()
    finite = (u & 0x7F800000) != 0x7F800000
    v = u[finite]
    u[finite] = (v + np.uint32(0x7FFF) + ((v >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return u.view(np.float32)


def tf32(x: np.ndarray) -> np.ndarray:
    """cvt.rna.tf32.f32 applied elementwise."""
    u = f32(x).view(np.uint32).copy()
    finite = (u & 0x7F800000) != 0x7F800000
    u[finite] = (u[finite] + np.uint32(0x1000)) & np.uint32(0xFFFFE000)
    return u.view(np.float32)


def ssim_window() -> np.ndarray:
    w = np.zeros(11, np.float32)
    lib().oracle_ssim_window(w)
    return w


def project_forward(means, scales, quats, opacities, world_to_camera, fx, fy, cx, cy, width, height,
                    near_plane=NEAR_PLANE, low_pass=LOW_PASS, fov_scale=FOV_SCALE):
    """projection.cu:80-111.  Returns means2D [N,2], depths [N], radii [N], conics [N,3]."""
    means, scales, quats = f32(means), f32(scales), f32(quats)
    n = means.shape[0]
    out = (np.zeros((n, 2), np.float32), np.zeros(n, np.float32), np.zeros(n, np.float32), np.zeros((n, 3), np.float32))
    lib().oracle_project_forward(n, means, scales, quats, f32(opacities).reshape(-1), f32(world_to_camera),
                                 fx, fy, cx, cy, width, height, near_plane, low_pass, fov_scale, *out)
    return out


def project_backward(grad_means2D, grad_conics, means, scales, quats, world_to_camera, fx, fy, cx, cy, width, height,
                     near_plane=NEAR_PLANE, low_pass=LOW_PASS, fov_scale=FOV_SCALE):
    """projection.cu:114-197.  Returns grad means [N,3], scales [N,3], quats [N,4]."""
    means, scales, quats = f32(means), f32(scales), f32(quats)
    n = means.shape[0]
    gm, gs, gq = np.zeros((n, 3), np.float32), np.zeros((n, 3), np.float32), np.zeros((n, 4), np.float32)
    lib().oracle_project_backward(n, f32(grad_means2D), f32(grad_conics), means, scales, quats, f32(world_to_camera),
                                  fx, fy, cx, cy, width, height, near_plane, low_pass, fov_scale, gm, gs, gq)
    return gm, gs, gq


def eval_sh(sh_dc, sh_rest, dirs, degree, radii):
    """sh.cu:62-83."""
    n = f32(dirs).shape[0]
    rgb = np.zeros((n, 3), np.float32)
    lib().oracle_eval_sh_forward(n, degree, f32(sh_dc), f32(sh_rest), f32(dirs), f32(radii), rgb)
    return rgb


def eval_sh_backward(grad_rgb, sh_dc, sh_rest, dirs, degree, radii):
    """The SH gradient of sh.cu:104-147, returned instead of consumed by Adam."""
    n = f32(dirs).shape[0]
    gdc, grest, gd = np.zeros((n, 1, 3), np.float32), np.zeros((n, 15, 3), np.float32), np.zeros((n, 3), np.float32)
    lib().oracle_eval_sh_backward(n, degree, f32(grad_rgb), f32(sh_dc), f32(sh_rest), f32(dirs), f32(radii),
                                  gdc, grest, gd)
    return gdc, grest, gd


def activate(log_scales, quats, logits):
    """The model's activations (utils/gaussian.py:73-98): (scales [N,3], unit quats [N,4], opacities)."""
    ls, q, lg = f32(log_scales), f32(quats), f32(logits)
    n = q.shape[0]
    scales, unit, opac = np.zeros((n, 3), np.float32), np.zeros((n, 4), np.float32), np.zeros(lg.shape, np.float32)
    lib().oracle_activate(n, ls, q, lg, scales, unit, opac)
    return scales, unit, opac


def activate_backward(log_scales, quats, logits, grad_scales, grad_unit_quats, grad_opacities=None):
    """Chain rule of activate: (dL/dlog_scales, dL/dquats, dL/dlogits)."""
    ls, q, lg = f32(log_scales), f32(quats), f32(logits)
    n = q.shape[0]
    gls, gq, glg = np.zeros((n, 3), np.float32), np.zeros((n, 4), np.float32), np.zeros(lg.shape, np.float32)
    gop = None if grad_opacities is None else f32(grad_opacities)
    lib().oracle_activate_backward(n, ls, q, lg, f32(grad_scales), f32(grad_unit_quats),
                                   None if gop is None else gop.ctypes.data, gls, gq, glg)
    return gls, gq, glg


def view_dirs(means, camera_center):
    """Viewing directions of the reference's Gaussian.colors (utils/gaussian.py:110):
    torch.nn.functional.normalize(means - camera_center, dim=-1) = x / max(|x|, 1e-12), in float32 with
    one rounding per operation and the squares summed x, y, z in order.  Returns (dirs [N,3], the
    divisor s [N])."""
    x = f32(means) - f32(camera_center).reshape(1, 3)
    s = np.sqrt(x[:, 0] * x[:, 0] + x[:, 1] * x[:, 1] + x[:, 2] * x[:, 2])
    s = np.maximum(s, np.float32(1e-12)).astype(np.float32)
    return (x / s[:, None]).astype(np.float32), s


def view_dirs_backward(grad_dirs, dirs, s):
    """dL/dmeans of view_dirs from dL/ddirs: (g - dir (dir . g)) / s above the 1e-12 clamp, g / s at it
    (the derivative of x / |x|; at the clamp the divisor is a constant)."""
    g, d = f32(grad_dirs), f32(dirs)
    dot = d[:, 0] * g[:, 0] + d[:, 1] * g[:, 1] + d[:, 2] * g[:, 2]
    above = (s > np.float32(1e-12))[:, None]
    out = np.where(above, (g - d * dot[:, None]) / s[:, None], g / s[:, None])
    return out.astype(np.float32)


def adam(p, m, v, g, step, lr, beta1, beta2, eps):
    """sh.cu:86-102, in place on copies; returns (p, m, v)."""
    p, m, v = f32(p).copy(), f32(m).copy(), f32(v).copy()
    lib().oracle_adam(p.size, p.reshape(-1), m.reshape(-1), v.reshape(-1), f32(g).reshape(-1), step, lr, beta1, beta2,
                      float(np.float32(1.0 - beta1)), float(np.float32(1.0 - beta2)), eps)
    return p, m, v


def tile_grid(width: int, height: int) -> tuple[int, int]:
    return (width + TILE - 1) // TILE, (height + TILE - 1) // TILE


def bin_gaussians(means2D, depths, radii, conics, opacities, width, height, origin_y=0):
    """forward.cu:13-139 plus the stable radix sort (forward.cu:363-394).  origin_y (a multiple of 16):
    bin the band of `height` rows starting at that row of a taller view (means2D in its pixels).

    Returns (tiles_touched [N] i32, keys_sorted [Dups] u64, values_sorted [Dups] i32, ranges [T,2] i32)."""
    args = [f32(means2D), f32(depths).reshape(-1), f32(radii).reshape(-1), f32(conics), f32(opacities).reshape(-1)]
    n = args[1].shape[0]
    tx, ty = tile_grid(width, height)
    touched = np.zeros(max(n, 1), np.int32)
    total = lib().oracle_bin(n, *args, width, height, int(origin_y), 0, None, None, None, _ptr(touched))
    keys = np.zeros(max(total, 1), np.uint64)
    vals = np.zeros(max(total, 1), np.int32)
    ranges = np.zeros((tx * ty, 2), np.int32)
    lib().oracle_bin(n, *args, width, height, int(origin_y), total, _ptr(keys), _ptr(vals), _ptr(ranges), None)
    return touched[:n], keys[:total], vals[:total], ranges


def render_forward(ranges, values, means2D, conics, colors, opacities, width, height, background=None,
                   features=None, tf32_round=False, split_bf16=False, origin_y=0):
    """forward.cu:141-237 (RGB) and features.cu:116-282 (features) over the binned lists.

    Feature products are exact by default; tf32_round rounds weights and features like
    cvt.rna.tf32 (the reference's tensor-core blend), split_bf16 forms them as hi*hi + hi*lo + lo*hi
    of bf16 halves (this library's tensor-core blend).  Sums are in double either way.
    Returns (image [H,W,3] or None, final_T [H,W], n_contrib [H,W] i32, feature_image or None)."""
    p = height * width
    image = np.zeros((height, width, 3), np.float32) if colors is not None else None
    final_T = np.zeros((height, width), np.float32)
    n_contrib = np.zeros((height, width), np.int32)
    ch = 0 if features is None else f32(features).shape[1]
    feat = np.zeros((height, width, ch), np.float32) if features is not None else None
    colors_a = None if colors is None else f32(colors)
    bg = None if background is None else f32(background)
    feats = None if features is None else f32(features)
    lib().oracle_render_forward(width, height, int(origin_y), np.ascontiguousarray(ranges, np.int32).reshape(-1),
                                np.ascontiguousarray(values, np.int32).reshape(-1), f32(means2D), f32(conics),
                                _ptr(colors_a), f32(opacities).reshape(-1), _ptr(bg), ch, _ptr(feats),
                                2 if split_bf16 else int(bool(tf32_round)), _ptr(image), _ptr(final_T),
                                _ptr(n_contrib), _ptr(feat))
    del p
    return image, final_T, n_contrib, feat


def render_backward(ranges, values, means2D, conics, colors, opacities, width, height, final_T, n_contrib,
                    grad_image=None, background=None, features=None, grad_features=None, origin_y=0):
    """backward.cu:7-164 and features.cu:350-542.  Returns float64 grads
    (means2D [N,2], conics [N,3], colors [N,3], opacities [N,1], features [N,C] or None)."""
    n = f32(means2D).shape[0]
    gm, gc = np.zeros((n, 2)), np.zeros((n, 3))
    gcol, go = np.zeros((n, 3)), np.zeros((n, 1))
    ch = 0 if features is None else f32(features).shape[1]
    gf = np.zeros((n, ch)) if features is not None else None
    bg = f32(background if background is not None else np.zeros(3))
    keep = [f32(colors) if colors is not None else None, bg,
            f32(grad_image) if grad_image is not None else None,
            f32(features) if features is not None else None,
            f32(grad_features) if grad_features is not None else None]
    lib().oracle_render_backward(width, height, int(origin_y), np.ascontiguousarray(ranges, np.int32).reshape(-1),
                                 np.ascontiguousarray(values, np.int32).reshape(-1), f32(means2D), f32(conics),
                                 _ptr(keep[0]), f32(opacities).reshape(-1), _ptr(keep[1]), f32(final_T),
                                 np.ascontiguousarray(n_contrib, np.int32), _ptr(keep[2]), ch, _ptr(keep[3]),
                                 _ptr(keep[4]), gm, gc, gcol, go, _ptr(gf))
    return gm, gc, gcol, go, gf


def ssim_forward(rendered, gt):
    """ssim.cu:208-262.  Returns (map, d_mu, d_aa, d_ab), each [H,W,3]."""
    a, b = f32(rendered), f32(gt)
    h, w = a.shape[:2]
    outs = [np.zeros_like(a) for _ in range(4)]
    lib().oracle_ssim_forward(h, w, a, b, *outs)
    return tuple(outs)


def ssim_backward(grad_mean, rendered, gt, d_mu, d_aa, d_ab):
    """ssim.cu:264-303."""
    a = f32(rendered)
    h, w = a.shape[:2]
    out = np.zeros_like(a)
    lib().oracle_ssim_backward(h, w, float(grad_mean), a, f32(gt), f32(d_mu), f32(d_aa), f32(d_ab), out)
    return out


def rasterize(means2D, depths, radii, conics, colors, opacities, width, height, background=None, features=None,
              tf32_round=False, origin_y=0):
    """Binning + blend in one call: the oracle's counterpart of the reference's rasterize (+ features).
    origin_y: the band of `height` rows starting at that row of a taller view."""
    touched, keys, values, ranges = bin_gaussians(means2D, depths, radii, conics, opacities, width, height, origin_y)
    image, final_T, n_contrib, feat = render_forward(ranges, values, means2D, conics, colors, opacities, width, height,
                                                     background, features, tf32_round, origin_y=origin_y)
    return {"tiles_touched": touched, "keys": keys, "values": values, "ranges": ranges, "image": image,
            "final_T": final_T, "n_contrib": n_contrib, "features": feat}

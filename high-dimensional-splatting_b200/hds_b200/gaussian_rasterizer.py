"""Drop-in replacement for the reference's ``gaussian_rasterizer`` torch extension.

Exports the ten entry points of gaussian_splatting/rasterizer/bindings.cpp:4-43 with the same
argument order, tensor layouts, return tuples and error messages, implemented on libhds_b200.so.
Outputs are allocated with torch's caching allocator on the inputs' device and all work is queued
on the current CUDA stream.  Additive entry points serve this package's own autograd layer:
``rasterize_with_features`` (one walk producing RGB and features), ``rasterize_backward_fused`` (one
walk for both backward passes), ``eval_sh_backward`` (plain SH gradients, for data-parallel training
that all-reduces them) and the ``*_into`` forms that add a gradient into a caller's buffer.

Every binning, blend and backward call also takes ``origin_y`` (keyword, default 0): the full
image's row at which the given image's row 0 lies, a multiple of 16.  With it an image of
``image_height`` rows is the band [origin_y, origin_y + image_height) of a taller view -- means2D in
full-image pixels -- and equals those rows of the full render bit for bit (the tile-row split).
"""
from __future__ import annotations

import ctypes

import torch

from .native import check, lib, ptr, stream_of

TILE = 16
_F32 = torch.float32
_I32 = torch.int32


def _check(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def _tiles(width: int, height: int) -> int:
    return ((width + TILE - 1) // TILE) * ((height + TILE - 1) // TILE)


def _bin(means2D, depths, radii, conics, colors, opacities, width, height, keep_keys=False, origin_y=0):
    """forward.cu:262-404: pack, count, scan, (host read), emit, sort, ranges.

    Returns (conic [N,4], color_opacity [N,4], values_sorted, tile_ranges [T,2], keys_sorted or None)."""
    n = means2D.shape[0]
    dev = means2D.device
    stream = stream_of(dev)
    conic = torch.empty(n, 4, dtype=_F32, device=dev)
    color_opacity = torch.empty(n, 4, dtype=_F32, device=dev)
    prep = torch.empty(lib.hds_rasterize_prepare_scratch_bytes(n), dtype=torch.uint8, device=dev)
    total = ctypes.c_int64(0)
    check(lib.hds_rasterize_prepare(n, ptr(means2D), ptr(depths), ptr(radii), ptr(conics), ptr(colors), ptr(opacities),
                                    width, height, int(origin_y), ptr(conic), ptr(color_opacity), ptr(prep), prep.numel(),
                                    ctypes.byref(total), stream))
    dups = total.value
    tiles = _tiles(width, height)
    if dups == 0:
        return conic, color_opacity, torch.empty(0, dtype=_I32, device=dev), \
            torch.zeros(tiles, 2, dtype=_I32, device=dev), (torch.empty(0, dtype=torch.int64, device=dev) if keep_keys else None)
    values = torch.empty(dups, dtype=_I32, device=dev)
    ranges = torch.empty(tiles, 2, dtype=_I32, device=dev)
    keys = torch.empty(dups, dtype=torch.int64, device=dev) if keep_keys else None
    scratch = torch.empty(lib.hds_rasterize_sort_scratch_bytes(n, dups, width, height), dtype=torch.uint8, device=dev)
    check(lib.hds_rasterize_sort(n, dups, width, height, ptr(prep), ptr(scratch), scratch.numel(), ptr(values),
                                 ptr(ranges), ptr(keys), stream))
    return conic, color_opacity, values, ranges, keys


def rasterize(means2D, depths, radii, conics, colors, opacities, background, image_width: int, image_height: int, *,
              origin_y: int = 0):
    """forward.cu:239-435.  Returns (image [H,W,3] view of [H,W,4], final_T [H,W], n_contrib [H,W],
    values_sorted [Dups], tile_ranges [T,2], conic [N,4], color_opacity [N,4])."""
    for t, name in ((means2D, "means2D"), (depths, "depths"), (radii, "radii"), (conics, "conics"),
                    (colors, "colors"), (opacities, "opacities"), (background, "background")):
        _check(t, name)
    width, height = int(image_width), int(image_height)
    dev = means2D.device
    conic, color_opacity, values, ranges, _ = _bin(means2D, depths, radii, conics, colors, opacities, width, height,
                                                   origin_y=origin_y)
    if values.numel() == 0:
        return (background.reshape(1, 1, 3).expand(height, width, 3).contiguous(),
                torch.ones(height, width, dtype=_F32, device=dev), torch.zeros(height, width, dtype=_I32, device=dev),
                values, ranges, conic, color_opacity)
    out = torch.empty(height, width, 4, dtype=_F32, device=dev)
    final_T = torch.empty(height, width, dtype=_F32, device=dev)
    n_contrib = torch.empty(height, width, dtype=_I32, device=dev)
    check(lib.hds_render_forward(width, height, int(origin_y), ptr(ranges), ptr(values), ptr(means2D), ptr(conic),
                                 ptr(color_opacity),
                                 ptr(background), ptr(out), ptr(final_T), ptr(n_contrib), stream_of(dev)))
    return out[..., :3], final_T, n_contrib, values, ranges, conic, color_opacity


def rasterize_with_features(means2D, depths, radii, conics, colors, opacities, background, features,
                            image_width: int, image_height: int, *, origin_y: int = 0):
    """rasterize + rasterize_features in one walk of the sorted lists (the RGB image is a by-product of
    the feature pass).  Returns (image, feature_image, final_T, n_contrib, values_sorted, tile_ranges,
    conic, color_opacity); final_T / n_contrib serve both images' backward passes."""
    for t, name in ((means2D, "means2D"), (depths, "depths"), (radii, "radii"), (conics, "conics"),
                    (colors, "colors"), (opacities, "opacities"), (background, "background")):
        _check(t, name)
    if not (features.is_cuda and features.is_contiguous() and features.dtype == _F32):
        raise RuntimeError("features must be a contiguous float32 CUDA tensor")
    width, height = int(image_width), int(image_height)
    dev = means2D.device
    n, d = features.shape
    conic, color_opacity, values, ranges, _ = _bin(means2D, depths, radii, conics, colors, opacities, width, height,
                                                   origin_y=origin_y)
    out = torch.empty(height, width, 4, dtype=_F32, device=dev)
    feature_image = torch.empty(height, width, d, dtype=_F32, device=dev)
    final_T = torch.empty(height, width, dtype=_F32, device=dev)
    n_contrib = torch.empty(height, width, dtype=_I32, device=dev)
    check(lib.hds_render_features_forward(n, d, width, height, int(origin_y), ptr(ranges), ptr(values), ptr(means2D),
                                          ptr(conic),
                                          ptr(color_opacity), ptr(features), ptr(background), ptr(feature_image),
                                          ptr(final_T), ptr(n_contrib), ptr(out), stream_of(dev)))
    return out[..., :3], feature_image, final_T, n_contrib, values, ranges, conic, color_opacity


def render_binned_with_features(values_sorted, tile_ranges, means2D, conic, color_opacity, features, background,
                                image_width: int, image_height: int, *, origin_y: int = 0):
    """The fused RGB + feature blend over lists binned earlier (values_sorted, tile_ranges of an image of
    this size and origin) and packed conic / color_opacity rows; no counterpart in the reference.  The
    gaussian ids in values_sorted index means2D, conic, color_opacity and features, which may be any
    compact subset of a scene's gaussians.  Returns (image [H,W,3], feature_image [H,W,D], final_T,
    n_contrib)."""
    if not (features.is_cuda and features.is_contiguous() and features.dtype == _F32):
        raise RuntimeError("features must be a contiguous float32 CUDA tensor")
    width, height = int(image_width), int(image_height)
    dev = features.device
    n, d = features.shape
    out = torch.empty(height, width, 4, dtype=_F32, device=dev)
    feature_image = torch.empty(height, width, d, dtype=_F32, device=dev)
    final_T = torch.empty(height, width, dtype=_F32, device=dev)
    n_contrib = torch.empty(height, width, dtype=_I32, device=dev)
    check(lib.hds_render_features_forward(n, d, width, height, int(origin_y), ptr(tile_ranges), ptr(values_sorted),
                                          ptr(means2D), ptr(conic), ptr(color_opacity), ptr(features),
                                          ptr(background), ptr(feature_image), ptr(final_T), ptr(n_contrib), ptr(out),
                                          stream_of(dev)))
    return out[..., :3], feature_image, final_T, n_contrib


def rasterize_backward(grad_image, means2D, conic, color_opacity, values_sorted, tile_ranges, final_transmittance,
                       n_contrib, background, image_width: int, image_height: int, *, origin_y: int = 0):
    """backward.cu:166-226.  Returns (dL/dmeans2D [N,2], dL/dconics [N,3], dL/dcolors [N,3], dL/dopacities [N,1])."""
    for t, name in ((grad_image, "grad_image"), (means2D, "means2D"), (conic, "conic"),
                    (color_opacity, "color_opacity"), (values_sorted, "values_sorted"), (tile_ranges, "tile_ranges"),
                    (final_transmittance, "final_transmittance"), (n_contrib, "n_contrib"), (background, "background")):
        _check(t, name)
    n = means2D.shape[0]
    dev = means2D.device
    gm = torch.empty(n, 2, dtype=_F32, device=dev)
    gc = torch.empty(n, 3, dtype=_F32, device=dev)
    gcol = torch.empty(n, 3, dtype=_F32, device=dev)
    go = torch.empty(n, 1, dtype=_F32, device=dev)
    check(lib.hds_render_backward(n, int(image_width), int(image_height), int(origin_y), ptr(grad_image), ptr(means2D),
                                  ptr(conic),
                                  ptr(color_opacity), ptr(values_sorted), ptr(tile_ranges), ptr(final_transmittance),
                                  ptr(n_contrib), ptr(background), ptr(gm), ptr(gc), ptr(gcol), ptr(go),
                                  stream_of(dev)))
    return gm, gc, gcol, go


def rasterize_features(features, means2D, conic, color_opacity, values_sorted, tile_ranges, image_width: int,
                       image_height: int, *, origin_y: int = 0):
    """features.cu:299-346.  Returns (feature_image [H,W,D], final_T [H,W], n_contrib [H,W])."""
    if not (features.is_cuda and features.is_contiguous() and features.dtype == _F32):
        raise RuntimeError("features must be a contiguous float32 CUDA tensor")
    width, height = int(image_width), int(image_height)
    dev = features.device
    n, d = features.shape
    out = torch.empty(height, width, d, dtype=_F32, device=dev)
    final_T = torch.empty(height, width, dtype=_F32, device=dev)
    n_contrib = torch.empty(height, width, dtype=_I32, device=dev)
    check(lib.hds_render_features_forward(n, d, width, height, int(origin_y), ptr(tile_ranges), ptr(values_sorted),
                                          ptr(means2D),
                                          ptr(conic), ptr(color_opacity), ptr(features), None, ptr(out), ptr(final_T),
                                          ptr(n_contrib), None, stream_of(dev)))
    return out, final_T, n_contrib


def rasterize_features_backward(grad_output, features, means2D, conic, color_opacity, values_sorted, tile_ranges,
                                final_transmittance, n_contrib, image_width: int, image_height: int, slice_width: int, *,
                                origin_y: int = 0):
    """features.cu:561-616.  Returns (dL/dfeatures [N,D], dL/dmeans2D [N,2], dL/dconics [N,3], dL/dopacities [N,1])."""
    if not (grad_output.is_cuda and grad_output.is_contiguous()):
        raise RuntimeError("grad_output must be a contiguous CUDA tensor")
    n, d = features.shape
    dev = features.device
    gf = torch.empty(n, d, dtype=_F32, device=dev)
    gm = torch.empty(n, 2, dtype=_F32, device=dev)
    gc = torch.empty(n, 3, dtype=_F32, device=dev)
    go = torch.empty(n, 1, dtype=_F32, device=dev)
    check(lib.hds_render_features_backward(n, d, int(slice_width), int(image_width), int(image_height), int(origin_y),
                                           ptr(grad_output),
                                           ptr(features), ptr(means2D), ptr(conic), ptr(color_opacity),
                                           ptr(values_sorted), ptr(tile_ranges), ptr(final_transmittance),
                                           ptr(n_contrib), ptr(gf), ptr(gm), ptr(gc), ptr(go), stream_of(dev)))
    return gf, gm, gc, go


def rasterize_features_backward_into(grad_features, grad_output, features, means2D, conic, color_opacity,
                                     values_sorted, tile_ranges, final_transmittance, n_contrib, image_width: int,
                                     image_height: int, slice_width: int, *, origin_y: int = 0):
    """rasterize_features_backward that ADDS dL/dfeatures into grad_features ([N,D] fp32, contiguous)
    instead of returning a fresh tensor; no counterpart in the reference.  Returns (dL/dmeans2D,
    dL/dconics, dL/dopacities)."""
    if not (grad_output.is_cuda and grad_output.is_contiguous()):
        raise RuntimeError("grad_output must be a contiguous CUDA tensor")
    n, d = features.shape
    if not (grad_features.is_contiguous() and grad_features.dtype == _F32 and tuple(grad_features.shape) == (n, d)
            and grad_features.device == features.device):
        raise RuntimeError("grad_features must be a contiguous float32 tensor shaped like features")
    dev = features.device
    gm = torch.empty(n, 2, dtype=_F32, device=dev)
    gc = torch.empty(n, 3, dtype=_F32, device=dev)
    go = torch.empty(n, 1, dtype=_F32, device=dev)
    check(lib.hds_render_features_backward_accumulate(
        n, d, int(slice_width), int(image_width), int(image_height), int(origin_y), ptr(grad_output), ptr(features),
        ptr(means2D),
        ptr(conic), ptr(color_opacity), ptr(values_sorted), ptr(tile_ranges), ptr(final_transmittance),
        ptr(n_contrib), ptr(grad_features), ptr(gm), ptr(gc), ptr(go), stream_of(dev)))
    return gm, gc, go


def rasterize_backward_fused(grad_image, background, grad_feature_image, features, means2D, conic, color_opacity,
                             values_sorted, tile_ranges, final_transmittance, n_contrib, image_width: int,
                             image_height: int, grad_features_into=None, *, origin_y: int = 0,
                             half_tile_lists: bool = True):
    """The RGB and feature backward in one walk (no counterpart in the reference, which runs
    rasterize_backward and rasterize_features_backward).  grad_image may be None (no RGB terms).
    grad_features_into, if given, is an [N, D] fp32 buffer that dL/dfeatures is added to.
    half_tile_lists: at 256 and 512 channels, cut every half tile's list in one kernel ahead of the
    walk (a workspace of hds_backward_workspace_bytes); False lets each block cut its own.

    Returns (dL/dmeans2D [N,2], dL/dconics [N,3], dL/dcolors [N,3] or None, dL/dopacities [N,1],
    dL/dfeatures [N,D] or None when added into grad_features_into)."""
    if not (grad_feature_image.is_cuda and grad_feature_image.is_contiguous()):
        raise RuntimeError("grad_feature_image must be a contiguous CUDA tensor")
    if grad_image is not None and not grad_image.is_contiguous():
        raise RuntimeError("grad_image must be contiguous")
    n, d = features.shape
    dev = features.device
    if grad_features_into is not None:
        if not (grad_features_into.is_contiguous() and grad_features_into.dtype == _F32
                and tuple(grad_features_into.shape) == (n, d) and grad_features_into.device == dev):
            raise RuntimeError("grad_features_into must be a contiguous float32 tensor shaped like features")
        gf, accumulate = grad_features_into, 1
    else:
        gf, accumulate = torch.empty(n, d, dtype=_F32, device=dev), 0
    gm = torch.empty(n, 2, dtype=_F32, device=dev)
    gc = torch.empty(n, 3, dtype=_F32, device=dev)
    go = torch.empty(n, 1, dtype=_F32, device=dev)
    gcol = torch.empty(n, 3, dtype=_F32, device=dev) if grad_image is not None else None
    ws, ws_bytes = None, 0
    if half_tile_lists and d in (256, 512):
        ws_bytes = int(lib.hds_backward_workspace_bytes(values_sorted.numel(), int(image_width), int(image_height)))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    check(lib.hds_render_backward_fused(
        n, d, int(image_width), int(image_height), int(origin_y), ptr(grad_image) if grad_image is not None else None,
        ptr(background) if grad_image is not None else None, ptr(grad_feature_image), ptr(features), ptr(means2D),
        ptr(conic), ptr(color_opacity), ptr(values_sorted), ptr(tile_ranges), ptr(final_transmittance),
        ptr(n_contrib), ptr(gcol) if gcol is not None else None, ptr(gf), ptr(gm), ptr(gc), ptr(go), accumulate,
        ptr(ws), ws_bytes, stream_of(dev)))
    return gm, gc, gcol, go, (None if accumulate else gf)


def eval_sh(sh_dc, sh_rest, dirs, degree: int, radii):
    """sh.cu:157-168.  Returns rgb [N,3]."""
    n = sh_dc.shape[0]
    rgb = torch.empty(n, 3, dtype=_F32, device=sh_dc.device)
    check(lib.hds_eval_sh_forward(n, int(degree), ptr(sh_dc), ptr(sh_rest), ptr(dirs), ptr(radii), ptr(rgb),
                                  stream_of(sh_dc.device)))
    return rgb


def eval_sh_backward_adam(grad_rgb, sh_dc, sh_rest, dirs, degree: int, radii, m_dc, v_dc, m_rest, v_rest, step_dc,
                          step_rest, lr_dc: float, lr_rest: float, beta1: float, beta2: float, eps: float):
    """sh.cu:171-190: steps sh_dc / sh_rest and their Adam moments in place, returns dL/ddirs [N,3]."""
    n = sh_dc.shape[0]
    grad_dirs = torch.empty_like(dirs)
    check(lib.hds_eval_sh_backward_adam(n, int(degree), ptr(grad_rgb), ptr(sh_dc), ptr(sh_rest), ptr(dirs), ptr(radii),
                                        ptr(m_dc), ptr(v_dc), ptr(m_rest), ptr(v_rest), ptr(step_dc), ptr(step_rest),
                                        float(lr_dc), float(lr_rest), float(beta1), float(beta2), float(1.0 - beta1),
                                        float(1.0 - beta2), float(eps), ptr(grad_dirs), stream_of(sh_dc.device)))
    return grad_dirs


def eval_sh_backward(grad_rgb, sh_dc, sh_rest, dirs, degree: int, radii):
    """Plain SH backward: returns (dL/dsh_dc [N,1,3], dL/dsh_rest [N,15,3], dL/ddirs [N,3])."""
    n = sh_dc.shape[0]
    gdc = torch.empty_like(sh_dc)
    grest = torch.empty_like(sh_rest)
    gd = torch.empty_like(dirs)
    check(lib.hds_eval_sh_backward(n, int(degree), ptr(grad_rgb), ptr(sh_dc), ptr(sh_rest), ptr(dirs), ptr(radii),
                                   ptr(gdc), ptr(grest), ptr(gd), stream_of(sh_dc.device)))
    return gdc, grest, gd


def eval_sh_backward_into(grad_sh_dc, grad_sh_rest, grad_rgb, sh_dc, sh_rest, dirs, degree: int, radii):
    """Plain SH backward that adds dL/dsh_dc and dL/dsh_rest into the given contiguous float32 buffers
    (shaped like sh_dc and sh_rest); returns dL/ddirs [N,3]."""
    n = sh_dc.shape[0]
    for name, buf, like in (("grad_sh_dc", grad_sh_dc, sh_dc), ("grad_sh_rest", grad_sh_rest, sh_rest)):
        if buf.shape != like.shape or buf.dtype != _F32 or not buf.is_contiguous() or buf.device != like.device:
            raise ValueError(f"{name} must be a contiguous float32 tensor of shape {tuple(like.shape)}")
    gd = torch.empty_like(dirs)
    check(lib.hds_eval_sh_backward_accumulate(n, int(degree), ptr(grad_rgb), ptr(sh_dc), ptr(sh_rest), ptr(dirs),
                                              ptr(radii), ptr(grad_sh_dc), ptr(grad_sh_rest), ptr(gd),
                                              stream_of(sh_dc.device)))
    return gd


def eval_sh_view(sh_dc, sh_rest, means, camera_center, degree: int, radii):
    """eval_sh of the directions normalize(means - camera_center) formed in the kernel (the reference's
    Gaussian.colors, utils/gaussian.py:100-112, in one launch).  camera_center: [3] on the device."""
    n = sh_dc.shape[0]
    rgb = torch.empty(n, 3, dtype=_F32, device=sh_dc.device)
    check(lib.hds_eval_sh_forward_view(n, int(degree), ptr(sh_dc), ptr(sh_rest), ptr(means), ptr(camera_center),
                                       ptr(radii), ptr(rgb), stream_of(sh_dc.device)))
    return rgb


def eval_sh_view_backward(grad_rgb, sh_dc, sh_rest, means, camera_center, degree: int, radii, into=None):
    """Backward of eval_sh_view: (dL/dsh_dc, dL/dsh_rest, dL/dmeans).  With into = (grad_sh_dc,
    grad_sh_rest, grad_means), contiguous float32 buffers shaped like sh_dc, sh_rest and means, the
    three gradients are added to them instead, and those buffers are returned."""
    n = sh_dc.shape[0]
    if into is None:
        bufs, accumulate = (torch.empty_like(sh_dc), torch.empty_like(sh_rest), torch.empty_like(means)), 0
    else:
        bufs, accumulate = tuple(into), 1
        for name, buf, like in zip(("grad_sh_dc", "grad_sh_rest", "grad_means"), bufs, (sh_dc, sh_rest, means)):
            if buf.shape != like.shape or buf.dtype != _F32 or not buf.is_contiguous() or buf.device != like.device:
                raise ValueError(f"{name} must be a contiguous float32 tensor of shape {tuple(like.shape)}")
    check(lib.hds_eval_sh_backward_view(n, int(degree), ptr(grad_rgb), ptr(sh_dc), ptr(sh_rest), ptr(means),
                                        ptr(camera_center), ptr(radii), ptr(bufs[0]), ptr(bufs[1]), ptr(bufs[2]),
                                        accumulate, stream_of(sh_dc.device)))
    return bufs


def project_gaussians(means, scales, quats, opacities, world_to_camera, fx: float, fy: float, cx: float, cy: float,
                      width: int, height: int, near_plane: float, low_pass: float, fov_scale: float):
    """projection.cu:210-231.  Returns (means2D [N,2], depths [N], radii [N], conics [N,3])."""
    n = means.shape[0]
    dev = means.device
    pose = world_to_camera.contiguous()
    opac = opacities.contiguous()
    means2D = torch.empty(n, 2, dtype=_F32, device=dev)
    depths = torch.empty(n, dtype=_F32, device=dev)
    radii = torch.empty(n, dtype=_F32, device=dev)
    conics = torch.empty(n, 3, dtype=_F32, device=dev)
    check(lib.hds_project_forward(n, ptr(means), ptr(scales), ptr(quats), ptr(opac), ptr(pose), float(fx), float(fy),
                                  float(cx), float(cy), int(width), int(height), float(near_plane), float(low_pass),
                                  float(fov_scale), ptr(means2D), ptr(depths), ptr(radii), ptr(conics), stream_of(dev)))
    return means2D, depths, radii, conics


def project_gaussians_backward(grad_means2D, grad_conics, means, scales, quats, world_to_camera, fx: float, fy: float,
                               cx: float, cy: float, width: int, height: int, near_plane: float, low_pass: float,
                               fov_scale: float):
    """projection.cu:234-253.  Returns (dL/dmeans [N,3], dL/dscales [N,3], dL/dquats [N,4])."""
    n = means.shape[0]
    dev = means.device
    pose = world_to_camera.contiguous()
    gm = torch.empty_like(means)
    gs = torch.empty_like(scales)
    gq = torch.empty_like(quats)
    check(lib.hds_project_backward(n, ptr(grad_means2D), ptr(grad_conics), ptr(means), ptr(scales), ptr(quats), ptr(pose),
                                   float(fx), float(fy), float(cx), float(cy), int(width), int(height),
                                   float(near_plane), float(low_pass), float(fov_scale), ptr(gm), ptr(gs), ptr(gq),
                                   stream_of(dev)))
    return gm, gs, gq


def project_gaussians_raw(means, log_scales, quats, opacity_logits, world_to_camera, fx: float, fy: float, cx: float,
                          cy: float, width: int, height: int, near_plane: float, low_pass: float, fov_scale: float):
    """project_gaussians of the model's raw parameters, activated in the kernel (exp of the log-scales,
    normalised quats, sigmoid of the opacity logits).  Returns (means2D [N,2], depths [N], radii [N],
    conics [N,3], opacities shaped like opacity_logits)."""
    n = means.shape[0]
    dev = means.device
    pose = world_to_camera.contiguous()
    logits = opacity_logits.contiguous()
    means2D = torch.empty(n, 2, dtype=_F32, device=dev)
    depths = torch.empty(n, dtype=_F32, device=dev)
    radii = torch.empty(n, dtype=_F32, device=dev)
    conics = torch.empty(n, 3, dtype=_F32, device=dev)
    opacities = torch.empty_like(logits)
    check(lib.hds_project_forward_raw(n, ptr(means), ptr(log_scales), ptr(quats), ptr(logits), ptr(pose), float(fx),
                                      float(fy), float(cx), float(cy), int(width), int(height), float(near_plane),
                                      float(low_pass), float(fov_scale), ptr(means2D), ptr(depths), ptr(radii),
                                      ptr(conics), ptr(opacities), stream_of(dev)))
    return means2D, depths, radii, conics, opacities


def project_gaussians_raw_backward(grad_means2D, grad_conics, grad_opacities, means, log_scales, quats, opacity_logits,
                                   world_to_camera, fx: float, fy: float, cx: float, cy: float, width: int,
                                   height: int, near_plane: float, low_pass: float, fov_scale: float, into=None):
    """Backward of project_gaussians_raw: (dL/dmeans, dL/dlog_scales, dL/dquats, dL/dopacity_logits).
    grad_opacities may be None.  With into = four contiguous float32 buffers shaped like the raw
    parameters, the gradients are added to them instead, and those buffers are returned."""
    n = means.shape[0]
    dev = means.device
    pose = world_to_camera.contiguous()
    like = (means, log_scales, quats, opacity_logits)
    if into is None:
        bufs, accumulate = tuple(torch.empty_like(t) for t in like), 0
    else:
        bufs, accumulate = tuple(into), 1
        for name, buf, t in zip(("grad_means", "grad_log_scales", "grad_quats", "grad_opacity_logits"), bufs, like):
            if buf.shape != t.shape or buf.dtype != _F32 or not buf.is_contiguous() or buf.device != t.device:
                raise ValueError(f"{name} must be a contiguous float32 tensor of shape {tuple(t.shape)}")
    gop = None if grad_opacities is None else grad_opacities.contiguous()
    check(lib.hds_project_backward_raw(n, ptr(grad_means2D), ptr(grad_conics), ptr(gop) if gop is not None else None,
                                       ptr(means), ptr(log_scales), ptr(quats), ptr(opacity_logits), ptr(pose),
                                       float(fx), float(fy), float(cx), float(cy), int(width), int(height),
                                       float(near_plane), float(low_pass), float(fov_scale), ptr(bufs[0]),
                                       ptr(bufs[1]), ptr(bufs[2]), ptr(bufs[3]), accumulate, stream_of(dev)))
    return bufs


def ssim_forward(rendered, gt):
    """ssim.cu:306-338.  Returns (ssim_map, d_mu, d_aa, d_ab), each [H,W,3]."""
    if not (rendered.is_cuda and gt.is_cuda):
        raise RuntimeError("ssim inputs must be CUDA tensors")
    if not (rendered.is_contiguous() and gt.is_contiguous()):
        raise RuntimeError("ssim inputs must be contiguous")
    if not (rendered.dim() == 3 and rendered.shape[2] == 3 and rendered.shape == gt.shape):
        raise RuntimeError("ssim inputs must both be [H, W, 3]")
    h, w = rendered.shape[:2]
    outs = [torch.empty_like(rendered) for _ in range(4)]
    check(lib.hds_ssim_forward(h, w, ptr(rendered), ptr(gt), *map(ptr, outs), stream_of(rendered.device)))
    return tuple(outs)


def ssim_backward(grad_mean, rendered, gt, d_mu, d_aa, d_ab):
    """ssim.cu:340-367.  Returns dL/drendered [H,W,3]."""
    h, w = rendered.shape[:2]
    grad = torch.empty_like(rendered)
    check(lib.hds_ssim_backward(h, w, ptr(grad_mean), ptr(rendered), ptr(gt), ptr(d_mu), ptr(d_aa), ptr(d_ab), ptr(grad),
                                stream_of(rendered.device)))
    return grad


def bin_gaussians(means2D, depths, radii, conics, opacities, image_width: int, image_height: int, *,
                  origin_y: int = 0):
    """The binning stage alone, with the sorted keys (for bit-exact checks against the oracle).
    Returns (keys_sorted int64 [Dups], values_sorted [Dups], tile_ranges [T,2])."""
    colors = torch.zeros(means2D.shape[0], 3, dtype=_F32, device=means2D.device)
    _, _, values, ranges, keys = _bin(means2D, depths, radii, conics, colors, opacities, int(image_width),
                                      int(image_height), keep_keys=True, origin_y=origin_y)
    return keys, values, ranges

"""Autograd layer over the blend: mirrors gaussian_splatting/rasterizer/__init__.py of the reference.

``_get_rasterizer()`` returns this package's ``gaussian_rasterizer`` module (the reference returns
its JIT-built extension), so a training loop written against the reference runs unchanged.
"""
from __future__ import annotations

import os
from types import ModuleType

import torch

from . import gaussian_rasterizer as _ext

# Channels each feature backward block owns (the reference's __init__.py:11-12, 158); None takes the
# widest slice, at most 128.  The slicing does not change the sums; it applies to 256 and 512 channels
# on the one-block kernel (256 by default, 512 with HDS_FEATURE_BWD_CLUSTER=0), where the RGB backward
# is a pass of its own.
FEATURE_SLICE_WIDTH: int | None = None


def _fused_backward(channels: int) -> bool:
    """Whether one walk carries both backward passes.  Up to 128 channels there is one channel slice,
    and the RGB terms ride in its walk.  The four-block clusters walk each pixel once, so the RGB terms
    ride along there too; they run 512 channels by default and 256 with HDS_FEATURE_BWD_CLUSTER=1 (=0:
    never).  With 256 or 512 channels on the one-block kernel, only the first of several slices would
    carry the RGB terms, and that lengthens its walk by more than the separate RGB pass costs."""
    if channels <= 128:
        return True
    switch = os.environ.get("HDS_FEATURE_BWD_CLUSTER")
    return switch == "1" or (switch != "0" and channels == 512)

# When true, the backward of a rasterize call whose features are a leaf that already holds a
# contiguous float32 .grad of its shape adds dL/dfeatures straight into that .grad (and hands
# autograd no gradient for it), instead of returning a fresh [N, D] tensor that autograd then adds.
# hds_b200.sh.eval_sh_grad does the same for sh_dc and sh_rest.  The flag is read when the forward
# runs.  For loops that accumulate several views into one gradient buffer.  Hooks registered on
# those tensors are not run for that gradient.  Off by default (the reference's behaviour).
ACCUMULATE_INTO_LEAF_GRAD: bool = False


class accumulate_leaf_grads:
    """Context manager that turns ACCUMULATE_INTO_LEAF_GRAD on for its body."""

    def __enter__(self):
        global ACCUMULATE_INTO_LEAF_GRAD
        self._old, ACCUMULATE_INTO_LEAF_GRAD = ACCUMULATE_INTO_LEAF_GRAD, True
        return self

    def __exit__(self, *exc):
        global ACCUMULATE_INTO_LEAF_GRAD
        ACCUMULATE_INTO_LEAF_GRAD = self._old
        return False


def _get_rasterizer() -> ModuleType:
    """The extension module with the reference's ten entry points (see gaussian_rasterizer.py)."""
    return _ext


class RasterizeGaussians(torch.autograd.Function):
    """Autograd node for tile binning and the alpha blend (the reference's __init__.py:57-165).

    With features, one walk of the sorted lists renders both images (the reference renders them in
    two passes); their shared transmittance and contributor counts feed both backward passes."""

    @staticmethod
    def forward(ctx, means2D, depths, radii, conics, colors, opacities, background, features, image_width,
                image_height, origin_y=0):
        ext = _get_rasterizer()
        width, height = int(image_width), int(image_height)
        ctx.image_size = (width, height)
        ctx.origin_y = o = int(origin_y)
        args = (means2D.contiguous(), depths.contiguous(), radii.contiguous(), conics.contiguous(),
                colors.contiguous(), opacities.contiguous(), background.contiguous())
        if features is None:
            image, final_T, n_contrib, values, ranges, conic, color_opacity = ext.rasterize(*args, width, height,
                                                                                            origin_y=o)
            ctx.save_for_backward(means2D, conic, color_opacity, values, ranges, final_T, n_contrib, background, None,
                                  None, None)
            return image
        ctx.features_leaf = features if (ACCUMULATE_INTO_LEAF_GRAD and features.is_leaf) else None
        features = features.contiguous()
        image, feature_image, final_T, n_contrib, values, ranges, conic, color_opacity = ext.rasterize_with_features(
            *args, features, width, height, origin_y=o)
        ctx.save_for_backward(means2D, conic, color_opacity, values, ranges, final_T, n_contrib, background, features,
                              final_T, n_contrib)
        return image, feature_image

    @staticmethod
    def backward(ctx, grad_image, grad_features=None):
        (means2D, conic, color_opacity, values, ranges, final_T, n_contrib, background, features, feature_T,
         feature_contrib) = ctx.saved_tensors
        width, height = ctx.image_size
        o = ctx.origin_y
        ext = _get_rasterizer()
        means2D = means2D.contiguous()
        # Frozen features still shape the geometry gradients (the reference's __init__.py:150-153).
        if features is not None and grad_features is not None and any(ctx.needs_input_grad[i] for i in (0, 3, 5, 7)):
            # One walk for both backward passes (the reference runs two); the forward was fused too.
            leaf = getattr(ctx, "features_leaf", None)
            target = leaf.grad if (leaf is not None and ctx.needs_input_grad[7]) else None
            if not (target is not None and target.is_contiguous() and target.dtype == torch.float32
                    and target.shape == features.shape and target.device == features.device
                    and target.data_ptr() % 16 == 0):
                target = None
            if _fused_backward(features.shape[1]):
                # The RGB terms ride along in the feature walk (one pass instead of two).
                with torch.cuda.nvtx.range("rasterize_backward_fused"):
                    grad_means2D, grad_conics, grad_colors, grad_opacities, grad_feats = ext.rasterize_backward_fused(
                        grad_image.contiguous() if grad_image is not None else None, background,
                        grad_features.contiguous(), features, means2D, conic, color_opacity, values, ranges,
                        feature_T, feature_contrib, width, height, grad_features_into=target, origin_y=o)
                if grad_colors is None:
                    grad_colors = torch.zeros(means2D.shape[0], 3, device=means2D.device)
            else:
                # One walk per 128-channel slice: the RGB backward is a pass of its own.
                if grad_image is None:
                    grad_image = torch.zeros(height, width, 3, device=means2D.device)
                with torch.cuda.nvtx.range("rasterize_backward"):
                    grad_means2D, grad_conics, grad_colors, grad_opacities = ext.rasterize_backward(
                        grad_image.contiguous(), means2D, conic, color_opacity, values, ranges, final_T, n_contrib,
                        background, width, height, origin_y=o)
                slice_width = FEATURE_SLICE_WIDTH or min(features.shape[1], 128)
                with torch.cuda.nvtx.range("rasterize_features_backward"):
                    if target is not None:
                        f_means2D, f_conics, f_opacities = ext.rasterize_features_backward_into(
                            target, grad_features.contiguous(), features, means2D, conic, color_opacity, values,
                            ranges, feature_T, feature_contrib, width, height, slice_width, origin_y=o)
                        grad_feats = None
                    else:
                        grad_feats, f_means2D, f_conics, f_opacities = ext.rasterize_features_backward(
                            grad_features.contiguous(), features, means2D, conic, color_opacity, values, ranges,
                            feature_T, feature_contrib, width, height, slice_width, origin_y=o)
                grad_means2D += f_means2D
                grad_conics += f_conics
                grad_opacities += f_opacities
            if not ctx.needs_input_grad[7]:
                grad_feats = None
            return (grad_means2D, None, None, grad_conics, grad_colors, grad_opacities, None, grad_feats, None, None,
                    None)
        if grad_image is None:
            grad_image = torch.zeros(height, width, 3, device=means2D.device)
        with torch.cuda.nvtx.range("rasterize_backward"):
            grad_means2D, grad_conics, grad_colors, grad_opacities = ext.rasterize_backward(
                grad_image.contiguous(), means2D, conic, color_opacity, values, ranges, final_T, n_contrib,
                background, width, height, origin_y=o)
        return grad_means2D, None, None, grad_conics, grad_colors, grad_opacities, None, None, None, None, None


def rasterize(means2D: torch.Tensor, depths: torch.Tensor, radii: torch.Tensor, conics: torch.Tensor,
              colors: torch.Tensor, opacities: torch.Tensor, image_width: int, image_height: int,
              background: torch.Tensor | None = None, features: torch.Tensor | None = None, *, origin_y: int = 0):
    """Alpha-blends projected gaussians into an image, front to back, on 16x16 tiles
    (the reference's __init__.py:168-211).

    Returns the [H, W, 3] image, or (image, [H, W, D] feature image) when features ([N, D], D one of
    32, 64, 128, 256 or 512) are given.  origin_y (a multiple of 16) renders the band of rows
    [origin_y, origin_y + image_height) of a taller view whose means2D these are."""
    n = means2D.shape[0]
    assert means2D.shape == (n, 2)
    assert depths.shape == (n,) and radii.shape == (n,)
    assert conics.shape == (n, 3) and colors.shape == (n, 3)
    assert opacities.shape == (n, 1)
    if background is None:
        background = torch.zeros(3, device=means2D.device, dtype=means2D.dtype)
    assert background.shape == (3,)
    assert features is None or (features.ndim == 2 and features.shape[0] == n)
    return RasterizeGaussians.apply(means2D, depths, radii, conics, colors, opacities, background, features,
                                    image_width, image_height, origin_y)

"""Projection autograd nodes: mirrors gaussian_splatting/rasterizer/projection.py of the reference, plus a
form that takes the model's raw parameters and applies their activations in the kernel."""
from __future__ import annotations

import torch

# projection.py:3-5 of the reference.
NEAR_PLANE = 0.2
LOW_PASS = 0.3
JACOBIAN_FOV_SCALE = 1.3


def quat_to_rotmat(quats: torch.Tensor) -> torch.Tensor:
    """[N, 4] unit quaternions (w, x, y, z) -> [N, 3, 3] rotation matrices."""
    w, x, y, z = quats.unbind(-1)
    return torch.stack([
        1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
        2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
        2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y),
    ], dim=-1).reshape(-1, 3, 3)


class ProjectGaussians(torch.autograd.Function):
    """EWA projection of 3-D gaussians to 2-D (projection.py:25-93 of the reference).

    Returns means2D [N, 2], depths [N] (sort keys only), radii [N] (0 = culled, no gradient) and
    conics [N, 3] (inverse 2-D covariance xx, xy, yy)."""

    @staticmethod
    def forward(ctx, means, scales, quats, opacities, world_to_camera, fx, fy, cx, cy, width, height):
        from .rasterizer import _get_rasterizer

        means, scales, quats = means.contiguous(), scales.contiguous(), quats.contiguous()
        outputs = _get_rasterizer().project_gaussians(
            means, scales, quats, opacities.detach(), world_to_camera, fx, fy, cx, cy, width, height,
            NEAR_PLANE, LOW_PASS, JACOBIAN_FOV_SCALE)
        ctx.save_for_backward(means, scales, quats, world_to_camera)
        ctx.camera = (fx, fy, cx, cy, width, height)
        ctx.mark_non_differentiable(outputs[1], outputs[2])
        return outputs

    @staticmethod
    def backward(ctx, grad_means2D, grad_depths, grad_radii, grad_conics):
        from .rasterizer import _get_rasterizer

        means, scales, quats, world_to_camera = ctx.saved_tensors
        if grad_means2D is None:
            grad_means2D = torch.zeros(means.shape[0], 2, device=means.device)
        if grad_conics is None:
            grad_conics = torch.zeros(means.shape[0], 3, device=means.device)
        with torch.cuda.nvtx.range("project_backward"):
            grads = _get_rasterizer().project_gaussians_backward(
                grad_means2D.contiguous(), grad_conics.contiguous(), means, scales, quats, world_to_camera,
                *ctx.camera, NEAR_PLANE, LOW_PASS, JACOBIAN_FOV_SCALE)
        return (*grads, None, None, None, None, None, None, None, None)


project_gaussians = ProjectGaussians.apply


class ProjectGaussiansRaw(torch.autograd.Function):
    """ProjectGaussians of the model's raw parameters, with the activations of the reference's
    utils/gaussian.py:73-98 (exp of the log-scales, normalised quaternions, sigmoid of the opacity
    logits) inside the projection kernels instead of torch glue.

    Returns means2D, depths, radii and conics as ProjectGaussians does, plus the activated opacities
    (shaped like the logits) for the blend; their gradient flows back to the logits.  Under
    hds_b200.rasterizer.accumulate_leaf_grads() (active during this forward), when the four raw
    parameters are leaves that hold float32 .grad buffers of their shapes, the backward adds the four
    gradients into those buffers and hands autograd none for them."""

    @staticmethod
    def forward(ctx, means, log_scales, quats, opacity_logits, world_to_camera, fx, fy, cx, cy, width, height):
        from . import rasterizer

        leaves = (means, log_scales, quats, opacity_logits)
        ctx.leaves = leaves if (rasterizer.ACCUMULATE_INTO_LEAF_GRAD and all(t.is_leaf for t in leaves)) else None
        means, log_scales, quats = means.contiguous(), log_scales.contiguous(), quats.contiguous()
        opacity_logits = opacity_logits.contiguous()
        outputs = rasterizer._get_rasterizer().project_gaussians_raw(
            means, log_scales, quats, opacity_logits, world_to_camera, fx, fy, cx, cy, width, height, NEAR_PLANE,
            LOW_PASS, JACOBIAN_FOV_SCALE)
        ctx.save_for_backward(means, log_scales, quats, opacity_logits, world_to_camera)
        ctx.camera = (fx, fy, cx, cy, width, height)
        ctx.mark_non_differentiable(outputs[1], outputs[2])
        return outputs

    @staticmethod
    def backward(ctx, grad_means2D, grad_depths, grad_radii, grad_conics, grad_opacities):
        from .rasterizer import _get_rasterizer
        from .sh import _grad_buffer

        means, log_scales, quats, logits, world_to_camera = ctx.saved_tensors
        if grad_means2D is None:
            grad_means2D = torch.zeros(means.shape[0], 2, device=means.device)
        if grad_conics is None:
            grad_conics = torch.zeros(means.shape[0], 3, device=means.device)
        args = (grad_means2D.contiguous(), grad_conics.contiguous(), grad_opacities, means, log_scales, quats, logits,
                world_to_camera, *ctx.camera, NEAR_PLANE, LOW_PASS, JACOBIAN_FOV_SCALE)
        none = (None,) * 7
        if ctx.leaves is not None and all(ctx.needs_input_grad[:4]):
            bufs = [_grad_buffer(leaf, like) for leaf, like in zip(ctx.leaves, (means, log_scales, quats, logits))]
            if all(b is not None for b in bufs):
                with torch.cuda.nvtx.range("project_backward"):
                    _get_rasterizer().project_gaussians_raw_backward(*args, into=bufs)
                return (None, None, None, None) + none
        with torch.cuda.nvtx.range("project_backward"):
            grads = _get_rasterizer().project_gaussians_raw_backward(*args)
        return (*grads, *none)


project_gaussians_raw = ProjectGaussiansRaw.apply

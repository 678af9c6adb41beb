"""SH colour autograd nodes: mirrors gaussian_splatting/utils/sh.py of the reference.

``eval_sh`` keeps the reference's contract: its backward steps sh_dc / sh_rest with the given Adam
in place and returns no SH gradient.  ``eval_sh_grad`` is the additive plain-gradient form used by
data-parallel training, where SH gradients must be all-reduced before any optimizer step.
"""
from __future__ import annotations

import torch

C0 = 0.28209479177387814


def num_sh_coeffs(degree: int) -> int:
    return (degree + 1) ** 2


def _adam_slot(optimizer: torch.optim.Adam, name: str):
    """Finds a named parameter's Adam group and state, creating the state like
    torch.optim.Adam(fused=True) and counting this step (sh.py:89-109 of the reference)."""
    group = next(g for g in optimizer.param_groups if g["name"] == name)
    param = group["params"][0]
    state = optimizer.state[param]
    if not state:
        state["step"] = torch.zeros((), dtype=torch.float32, device=param.device)
        state["exp_avg"] = torch.zeros_like(param, memory_format=torch.preserve_format)
        state["exp_avg_sq"] = torch.zeros_like(param, memory_format=torch.preserve_format)
    state["step"] += 1
    return param, group, state


class EvalSH(torch.autograd.Function):
    """RGB = max(0.5 + sum_j b_j(dir) w_j, 0) per gaussian, zero where culled; backward = fused Adam."""

    @staticmethod
    def forward(ctx, sh_dc, sh_rest, dirs, degree, radii, optimizer):
        from .rasterizer import _get_rasterizer

        sh_dc, sh_rest, dirs, radii = sh_dc.contiguous(), sh_rest.contiguous(), dirs.contiguous(), radii.contiguous()
        ctx.save_for_backward(dirs, radii)
        ctx.degree = degree
        ctx.optimizer = optimizer
        return _get_rasterizer().eval_sh(sh_dc, sh_rest, dirs, degree, radii)

    @staticmethod
    def backward(ctx, grad_rgb):
        from .rasterizer import _get_rasterizer

        if ctx.optimizer is None:
            raise RuntimeError("eval_sh backward needs the Adam that holds sh_dc and sh_rest, set model.sh_optimizer")
        dirs, radii = ctx.saved_tensors
        with torch.cuda.nvtx.range("sh_backward"):
            dc, dc_group, dc_state = _adam_slot(ctx.optimizer, "sh_dc")
            rest, rest_group, rest_state = _adam_slot(ctx.optimizer, "sh_rest")
            beta1, beta2 = dc_group["betas"]
            grad_dirs = _get_rasterizer().eval_sh_backward_adam(
                grad_rgb.contiguous(), dc.data, rest.data, dirs, ctx.degree, radii,
                dc_state["exp_avg"], dc_state["exp_avg_sq"], rest_state["exp_avg"], rest_state["exp_avg_sq"],
                dc_state["step"], rest_state["step"], dc_group["lr"], rest_group["lr"], beta1, beta2, dc_group["eps"])
        return None, None, grad_dirs, None, None, None


eval_sh = EvalSH.apply


def _grad_buffer(leaf, like):
    """leaf.grad when it can take an in-place add of a gradient shaped like `like`, else None."""
    g = leaf.grad
    if (g is not None and g.is_contiguous() and g.dtype == torch.float32 and g.shape == like.shape
            and g.device == like.device):
        return g
    return None


class EvalSHGrad(torch.autograd.Function):
    """Same colour as EvalSH; the backward returns dL/dsh_dc, dL/dsh_rest and dL/ddirs.

    Under hds_b200.rasterizer.accumulate_leaf_grads() (active during this forward), when sh_dc and
    sh_rest are leaves that already hold float32 .grad buffers of their shapes, the backward adds the
    SH gradients into those buffers and hands autograd none for them (hooks on the two tensors do not
    see that gradient)."""

    @staticmethod
    def forward(ctx, sh_dc, sh_rest, dirs, degree, radii):
        from . import rasterizer

        ctx.leaves = ((sh_dc, sh_rest) if (rasterizer.ACCUMULATE_INTO_LEAF_GRAD and sh_dc.is_leaf and sh_rest.is_leaf)
                      else None)
        sh_dc, sh_rest, dirs, radii = sh_dc.contiguous(), sh_rest.contiguous(), dirs.contiguous(), radii.contiguous()
        ctx.save_for_backward(sh_dc, sh_rest, dirs, radii)
        ctx.degree = degree
        return rasterizer._get_rasterizer().eval_sh(sh_dc, sh_rest, dirs, degree, radii)

    @staticmethod
    def backward(ctx, grad_rgb):
        from .rasterizer import _get_rasterizer

        sh_dc, sh_rest, dirs, radii = ctx.saved_tensors
        ext = _get_rasterizer()
        if ctx.leaves is not None and ctx.needs_input_grad[0] and ctx.needs_input_grad[1]:
            buf_dc, buf_rest = _grad_buffer(ctx.leaves[0], sh_dc), _grad_buffer(ctx.leaves[1], sh_rest)
            if buf_dc is not None and buf_rest is not None:
                gd = ext.eval_sh_backward_into(buf_dc, buf_rest, grad_rgb.contiguous(), sh_dc, sh_rest, dirs,
                                               ctx.degree, radii)
                return None, None, gd, None, None
        gdc, grest, gd = ext.eval_sh_backward(grad_rgb.contiguous(), sh_dc, sh_rest, dirs, ctx.degree, radii)
        return gdc, grest, gd, None, None


eval_sh_grad = EvalSHGrad.apply


class ViewColors(torch.autograd.Function):
    """RGB of every gaussian seen from camera_center: eval_sh of normalize(means - camera_center), with
    the normalisation inside the SH kernels (the reference's Gaussian.colors, utils/gaussian.py:100-112,
    runs it as torch glue).  The backward returns dL/dsh_dc, dL/dsh_rest, dL/dmeans and, when asked
    for, dL/dcamera_center = -sum dL/dmeans.

    Under hds_b200.rasterizer.accumulate_leaf_grads() (active during this forward), when sh_dc,
    sh_rest and means are leaves that hold float32 .grad buffers of their shapes and the camera centre
    needs no gradient, the backward adds its three gradients into those buffers and hands autograd
    none for them (hooks on the three tensors do not see that gradient)."""

    @staticmethod
    def forward(ctx, sh_dc, sh_rest, means, camera_center, degree, radii):
        from . import rasterizer

        leaves = (sh_dc, sh_rest, means)
        ctx.leaves = leaves if (rasterizer.ACCUMULATE_INTO_LEAF_GRAD and all(t.is_leaf for t in leaves)) else None
        sh_dc, sh_rest, means, radii = sh_dc.contiguous(), sh_rest.contiguous(), means.contiguous(), radii.contiguous()
        center = camera_center.detach().reshape(3).to(torch.float32).contiguous()
        ctx.center_shape, ctx.center_dtype = camera_center.shape, camera_center.dtype
        ctx.save_for_backward(sh_dc, sh_rest, means, center, radii)
        ctx.degree = degree
        return rasterizer._get_rasterizer().eval_sh_view(sh_dc, sh_rest, means, center, degree, radii)

    @staticmethod
    def backward(ctx, grad_rgb):
        from .rasterizer import _get_rasterizer

        sh_dc, sh_rest, means, center, radii = ctx.saved_tensors
        ext = _get_rasterizer()
        args = (grad_rgb.contiguous(), sh_dc, sh_rest, means, center, ctx.degree, radii)
        if ctx.leaves is not None and all(ctx.needs_input_grad[:3]) and not ctx.needs_input_grad[3]:
            bufs = [_grad_buffer(leaf, like) for leaf, like in zip(ctx.leaves, (sh_dc, sh_rest, means))]
            if all(b is not None for b in bufs):
                ext.eval_sh_view_backward(*args, into=bufs)
                return None, None, None, None, None, None
        gdc, grest, gmeans = ext.eval_sh_view_backward(*args)
        gcenter = None
        if ctx.needs_input_grad[3]:
            gcenter = (-gmeans.sum(dim=0)).reshape(ctx.center_shape).to(ctx.center_dtype)
        return gdc, grest, gmeans, gcenter, None, None


def view_colors(sh_dc, sh_rest, means, camera_center, degree: int, radii):
    """[N, 3] colours of the gaussians seen from camera_center [3] (zero where radii <= 0)."""
    return ViewColors.apply(sh_dc, sh_rest, means, camera_center, degree, radii)


def rgb_to_sh(rgb: torch.Tensor) -> torch.Tensor:
    """Inverts eval_sh at degree 0."""
    return (rgb - 0.5) / C0

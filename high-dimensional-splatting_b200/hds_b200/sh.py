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


class EvalSHGrad(torch.autograd.Function):
    """Same colour as EvalSH; the backward returns dL/dsh_dc, dL/dsh_rest and dL/ddirs."""

    @staticmethod
    def forward(ctx, sh_dc, sh_rest, dirs, degree, radii):
        from .rasterizer import _get_rasterizer

        sh_dc, sh_rest, dirs, radii = sh_dc.contiguous(), sh_rest.contiguous(), dirs.contiguous(), radii.contiguous()
        ctx.save_for_backward(sh_dc, sh_rest, dirs, radii)
        ctx.degree = degree
        return _get_rasterizer().eval_sh(sh_dc, sh_rest, dirs, degree, radii)

    @staticmethod
    def backward(ctx, grad_rgb):
        from .rasterizer import _get_rasterizer

        sh_dc, sh_rest, dirs, radii = ctx.saved_tensors
        gdc, grest, gd = _get_rasterizer().eval_sh_backward(grad_rgb.contiguous(), sh_dc, sh_rest, dirs, ctx.degree,
                                                            radii)
        return gdc, grest, gd, None, None


eval_sh_grad = EvalSHGrad.apply


def rgb_to_sh(rgb: torch.Tensor) -> torch.Tensor:
    """Inverts eval_sh at degree 0."""
    return (rgb - 0.5) / C0

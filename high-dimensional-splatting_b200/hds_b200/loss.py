"""Losses: mirrors gaussian_splatting/utils/loss.py of the reference (L1, PSNR, fused SSIM)."""
from __future__ import annotations

import torch


def l1_loss(rendered: torch.Tensor, gt: torch.Tensor) -> torch.Tensor:
    return (rendered - gt).abs().mean()


def psnr(rendered: torch.Tensor, gt: torch.Tensor) -> torch.Tensor:
    return -10.0 * torch.log10(((rendered - gt) ** 2).mean())


class FusedSSIM(torch.autograd.Function):
    """Mean SSIM with the per-pixel partials kept for the backward (loss.py:57-90 of the reference)."""

    @staticmethod
    def forward(ctx, rendered, gt):
        from .rasterizer import _get_rasterizer

        ssim_map, d_mu, d_aa, d_ab = _get_rasterizer().ssim_forward(rendered, gt)
        ctx.save_for_backward(rendered, gt, d_mu, d_aa, d_ab)
        return ssim_map.mean()

    @staticmethod
    def backward(ctx, grad_mean):
        from .rasterizer import _get_rasterizer

        rendered, gt, d_mu, d_aa, d_ab = ctx.saved_tensors
        grad = _get_rasterizer().ssim_backward(grad_mean.reshape(1).contiguous(), rendered, gt, d_mu, d_aa, d_ab)
        return grad, None


def ssim(rendered: torch.Tensor, gt: torch.Tensor, size: int = 11, sigma: float = 1.5) -> torch.Tensor:
    """Mean SSIM over every pixel and channel of two [H, W, 3] images, 11x11 window, sigma 1.5.

    Only the fused CUDA path exists: other windows, dtypes or CPU tensors raise."""
    if not (rendered.is_cuda and rendered.dtype == torch.float32 and size == 11 and sigma == 1.5):
        raise NotImplementedError("ssim runs on CUDA float32 [H, W, 3] images with the 11x11, sigma 1.5 window")
    return FusedSSIM.apply(rendered.contiguous(), gt.detach().contiguous())

"""B200 (sm_100a) rasterizer for high-dimensional gaussian splatting.

A drop-in for the hot path of alexkato29/high-dimensional-splatting: the same Python entry points
(rasterize, project_gaussians, eval_sh, ssim and the autograd nodes behind them) and the same
extension entry points (``_get_rasterizer()``), implemented on hand-written sm_100a kernels in
libhds_b200.so (C ABI: include/hds_b200.h).  Two additions fold the model's torch glue into those
kernels: project_gaussians_raw (the parameter activations) and view_colors (the view directions).
"""
from .projection import (JACOBIAN_FOV_SCALE, LOW_PASS, NEAR_PLANE, ProjectGaussians, ProjectGaussiansRaw,
                         project_gaussians, project_gaussians_raw, quat_to_rotmat)
from .rasterizer import FEATURE_SLICE_WIDTH, RasterizeGaussians, _get_rasterizer, accumulate_leaf_grads, rasterize
from .sh import view_colors

__all__ = ["rasterize", "project_gaussians", "project_gaussians_raw", "view_colors", "accumulate_leaf_grads",
           "RasterizeGaussians", "ProjectGaussians", "ProjectGaussiansRaw", "quat_to_rotmat", "_get_rasterizer",
           "FEATURE_SLICE_WIDTH", "NEAR_PLANE", "LOW_PASS", "JACOBIAN_FOV_SCALE"]

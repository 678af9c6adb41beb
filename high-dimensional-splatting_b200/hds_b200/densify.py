"""Densification on the device: the reference's GaussianModel.add_densification_stats and
densify_and_prune (utils/gaussian.py:143-296) over this package's flat parameter buffers.

The statistics are one kernel per view (hds_densify_stats).  densify_and_prune classifies the
gaussians with the reference's tests -- clone small gaussians whose mean 2-D gradient reaches the
threshold, split large ones into `into` children sampled inside them, prune transparent ones and,
once opacities have been reset, oversized ones -- and then writes the new population's parameters and
Adam moments with one kernel (hds_densify_apply) instead of an index / cat per tensor.  The new
population has the reference's row order: the surviving original rows, then the clones, then the
children (all first children, then all second children), and appended rows start with zero Adam
moments.  As in the reference, the statistics restart at zero afterwards.
"""
from __future__ import annotations

import ctypes

import torch

from .native import check, lib, ptr, stream_of
from .optim import FlatAdam

# The parameter tensors FlatAdam holds, in order, and their row widths (features last, optional).
LAYOUT = ("means", "log_scales", "quats", "opacity_logits", "sh_dc", "sh_rest")
SPLIT_CHILD, FRESH_STATE = 1, 2


class DensifyStats:
    """max_radii2D [n], grad_accum [n, 1], denom [n, 1] (the reference's _reset_stats)."""

    def __init__(self, n: int, device):
        self.max_radii2D = torch.zeros(n, device=device)
        self.grad_accum = torch.zeros(n, 1, device=device)
        self.denom = torch.zeros(n, 1, device=device)

    def add(self, grad_means2D: torch.Tensor, radii: torch.Tensor, width: int, height: int) -> None:
        """add_densification_stats (gaussian.py:143-160) in one kernel."""
        g = grad_means2D.contiguous()
        check(lib.hds_densify_stats(g.shape[0], ptr(g), ptr(radii.contiguous()), int(width), int(height),
                                    ptr(self.max_radii2D), ptr(self.grad_accum), ptr(self.denom),
                                    stream_of(g.device)))


def _rotmat(q: torch.Tensor) -> torch.Tensor:
    w, x, y, z = q.unbind(-1)
    return torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
                        2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
                        2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1).reshape(-1, 3, 3)


@torch.no_grad()
def densify_and_prune(opt: FlatAdam, stats: DensifyStats, grad_threshold: float, percent_dense: float,
                      min_opacity: float, extent: float, max_screen_size: float | None, into: int = 2,
                      normals: torch.Tensor | None = None, generator: torch.Generator | None = None):
    """Clones, splits and prunes the gaussians held by `opt` (a FlatAdam over LAYOUT [+ features]).

    normals: the [into * n_split, 3] standard-normal-times-std draws of the split children's offsets
    (the reference's torch.normal(0, stds)); drawn with `generator` when None.  Returns the new
    FlatAdam (same learning rates and step count) and fresh DensifyStats."""
    P = dict(zip(LAYOUT, opt.params))
    n = P["means"].shape[0]
    dev = P["means"].device
    scales = torch.exp(P["log_scales"])
    opac = torch.sigmoid(P["opacity_logits"])
    grads = torch.nan_to_num(stats.grad_accum / stats.denom.clamp_min(1)).squeeze(-1)
    # _clone (gaussian.py:194-208): the population becomes [old, clones].
    clone_idx = torch.nonzero((grads >= grad_threshold) & (scales.max(dim=1).values <= percent_dense * extent)).squeeze(1)
    p1_src = torch.cat([torch.arange(n, device=dev), clone_idx])
    p1_scales = scales[p1_src]
    padded = torch.cat([grads, torch.zeros(clone_idx.numel(), device=dev)])
    # _split (gaussian.py:210-244) over that population; its parents are removed.
    split_sel = (padded >= grad_threshold) & (p1_scales.max(dim=1).values > percent_dense * extent)
    split_p1 = torch.nonzero(split_sel).squeeze(1)
    stds = p1_scales[split_p1].repeat(into, 1)
    if normals is None:
        normals = torch.normal(torch.zeros_like(stds), stds, generator=generator)
    unit_q = torch.nn.functional.normalize(P["quats"][p1_src[split_p1]], dim=-1)
    offsets = torch.bmm(_rotmat(unit_q).repeat(into, 1, 1), normals.reshape(-1, 3, 1)).squeeze(-1)
    child_scales = torch.exp(torch.log(stds / (0.8 * into)))
    keep_p1 = ~split_sel
    p3_src = torch.cat([p1_src[keep_p1], p1_src[split_p1].repeat(into)])
    fresh = torch.cat([torch.arange(p1_src.numel(), device=dev)[keep_p1] >= n,
                       torch.ones(into * split_p1.numel(), dtype=torch.bool, device=dev)])
    child = torch.cat([torch.zeros(int(keep_p1.sum()), dtype=torch.bool, device=dev),
                       torch.ones(into * split_p1.numel(), dtype=torch.bool, device=dev)])
    p3_offsets = torch.cat([torch.zeros(int(keep_p1.sum()), 3, device=dev), offsets])
    p3_scales = torch.cat([p1_scales[keep_p1], child_scales])
    # The final prune (gaussian.py:181-188) over the new population; its 2-D radii statistics were
    # reset by the appends, so only the opacity and world-size tests can remove a row.
    prune = (opac[p3_src].squeeze(-1) < min_opacity)
    if max_screen_size is not None:
        prune |= p3_scales.max(dim=1).values > 0.1 * extent
    keep = torch.nonzero(~prune).squeeze(1)
    src = p3_src[keep].to(torch.int32).contiguous()
    flags = (child[keep].to(torch.uint8) * SPLIT_CHILD + fresh[keep].to(torch.uint8) * FRESH_STATE).contiguous()
    child_offset = p3_offsets[keep].contiguous()
    n_new = src.numel()
    widths = [p.shape[1:].numel() if p.dim() > 1 else 1 for p in opt.params]
    shapes = [(n_new,) + tuple(p.shape[1:]) for p in opt.params]
    total = sum(w * n_new for w in widths)
    new_flat = torch.empty(total, device=dev)
    new_m, new_v = torch.empty_like(new_flat), torch.empty_like(new_flat)
    w_arr = (ctypes.c_int * len(widths))(*widths)
    params = opt.flat[opt.head:opt.head + opt.n]  # the parameters, past any head reserve
    check(lib.hds_densify_apply(n, n_new, len(widths), w_arr, LAYOUT.index("means"), LAYOUT.index("log_scales"),
                                float(0.8 * into), ptr(src), ptr(flags), ptr(child_offset), ptr(params),
                                ptr(opt.exp_avg), ptr(opt.exp_avg_sq), ptr(new_flat), ptr(new_m), ptr(new_v),
                                stream_of(dev)))
    new_opt = FlatAdam.from_buffers(shapes, new_flat, new_m, new_v, opt.lrs, opt.step_count, opt.betas, opt.eps)
    return new_opt, DensifyStats(n_new, dev)

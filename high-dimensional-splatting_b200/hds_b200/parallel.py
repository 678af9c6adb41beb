"""Multi-GPU plumbing: data parallel over views, and one view split into tile-row bands.

The reference is single-GPU.  Two ways to use N GPUs of one node, one process per GPU:

* Views (data parallel): every rank holds a full replica of the gaussians and renders its own
  views; the per-gaussian gradients are summed over ranks with one all-reduce of a flat bucket.
* Tile rows (one large view): every rank projects all gaussians with the full camera (the
  projection's field-of-view clamp depends on the full image size) but bins and blends only a band
  of rows.  A band starting on a 16-row boundary is rendered as an image of its own with the 2-D
  means shifted up by the band's first row: its tiles coincide with the full image's tiles and
  conics, radii and opacities are unchanged, so band pixels match the full render up to the
  rounding of the shifted means.  Band gradients are partial sums over pixels; summing them over
  ranks gives the full-image gradient.
"""
from __future__ import annotations

import math

import torch

TILE = 16


def shard_views(n_views: int, rank: int, world: int) -> list[int]:
    """Round-robin assignment of view indices to ranks; every view lands on exactly one rank."""
    return list(range(rank, n_views, world))


def row_bands(height: int, world: int, row_weights: list[float] | None = None) -> list[tuple[int, int]]:
    """Splits [0, height) into `world` bands of whole tile rows, balanced by per-tile-row weights
    (e.g. the number of (tile, gaussian) pairs per tile row; uniform when None).  Every band holds at
    least one tile row, so `world` may not exceed the view's tile rows: ValueError otherwise."""
    rows = math.ceil(height / TILE)
    if world < 1 or world > rows:
        raise ValueError(f"{world} bands of a {height}-row view: 1 to {rows} (its tile rows) supported")
    w = list(row_weights) if row_weights is not None else [1.0] * rows
    assert len(w) == rows
    total = sum(w)
    bands, start, acc = [], 0, 0.0
    for r in range(world):
        if r == world - 1:
            end = rows
        else:
            target = total * (r + 1) / world
            end = start
            # Leave at least one tile row for every later band.
            while end < rows - (world - 1 - r) and (acc + w[end] <= target or end == start):
                acc += w[end]
                end += 1
        bands.append((start * TILE, min(end * TILE, height)))
        start = end
    return bands


def band_means(means2D: torch.Tensor, y0: int) -> torch.Tensor:
    """2-D means in the coordinates of a band whose first row is y0 (differentiable)."""
    assert y0 % TILE == 0, "bands must start on a tile row"
    return means2D - torch.tensor([0.0, float(y0)], dtype=means2D.dtype, device=means2D.device)


def render_band(rasterize_fn, means2D, depths, radii, conics, colors, opacities, width: int, y0: int, y1: int,
                background=None, features=None):
    """Rows [y0, y1) of the full render, as produced by `rasterize_fn` (hds_b200.rasterize)."""
    return rasterize_fn(band_means(means2D, y0), depths, radii, conics, colors, opacities, width, y1 - y0,
                        background, features)


class GradBucket:
    """One flat fp32 buffer holding the gradients of a list of parameters.

    attach() points every parameter's .grad at its slice, so autograd accumulates in place across
    views; all_reduce() then sums all gradients over ranks with a single collective."""

    def __init__(self, params: list[torch.Tensor], capacity: int = 0, offset: int = 0):
        """capacity: the flat buffer's length when it must exceed the parameters' (zero padding at
        the end, e.g. to split it evenly across ranks); offset: elements before the first parameter's
        slice (zero padding at the start)."""
        self.params = params
        total = sum(p.numel() for p in params)
        self.flat = torch.zeros(max(offset + total, capacity), dtype=torch.float32, device=params[0].device)
        self.views = []
        off = offset
        for p in params:
            self.views.append(self.flat[off:off + p.numel()].view_as(p))
            off += p.numel()
        self._side = None      # stream of zero_async
        self._pending = False  # a zero_async clear that the current stream has not waited for yet

    def attach(self) -> None:
        for p, v in zip(self.params, self.views):
            p.grad = v

    def zero(self) -> None:
        self.ready()
        self.flat.zero_()
        self.attach()

    def zero_async(self) -> None:
        """zero() on a side stream, so that the clear overlaps the work queued after it (the forward
        pass, which writes no gradient).  The clear starts once the current stream's earlier work is
        done; ready() makes the current stream wait for it and must run before anything writes or
        reads a gradient (the backward, all_reduce).  On a CPU bucket this is zero()."""
        if self.flat.device.type != "cuda":
            self.zero()
            return
        current = torch.cuda.current_stream(self.flat.device)
        if self._side is None:
            self._side = torch.cuda.Stream(self.flat.device)
        self._side.wait_stream(current)
        with torch.cuda.stream(self._side):
            self.flat.zero_()
        self._pending = True
        self.attach()

    def ready(self) -> None:
        """Makes the current stream wait for a clear started by zero_async (no-op otherwise)."""
        if self._pending:
            torch.cuda.current_stream(self.flat.device).wait_stream(self._side)
            self._pending = False

    def all_reduce(self, group=None) -> None:
        import torch.distributed as dist

        self.ready()
        dist.all_reduce(self.flat, group=group)
        for p, v in zip(self.params, self.views):
            if p.grad is None or p.grad.data_ptr() != v.data_ptr():
                raise RuntimeError("a gradient was re-allocated outside the bucket; call attach() before backward")

"""One view split into bands of tile rows across the ranks of a process group.

The tile-row form of data parallelism for a single large view (the benchmark's stress configuration:
4M gaussians, one 1920x1080 view, C = 512 features, on N GPUs of one node).  The reference is
single-GPU; this module is the multi-GPU plan built around its rasterizer:

* Geometry and SH (59 floats per gaussian) are replicated.  Every rank projects every gaussian with
  the full camera and evaluates its colour, then bins and renders only its band of tile rows with
  ``origin_y`` = the band's first row, so its pixels equal those rows of the full render bit for bit.
* The feature table (C floats per gaussian, the bulk of the model) is sharded: rank r owns the rows
  of one contiguous block of gaussians and their Adam state (FeatureShards).  Before rendering, each
  rank fetches the rows of the gaussians that can reach its band from their owners (all-to-all
  "dispatch"); after the backward it sends their gradients back, and each owner adds the
  contributions of every band (all-to-all "combine").  A gaussian that straddles a band boundary is
  reduced by its owner; a rank moves only the rows its band needs, not the table.
* The loss keeps the full image's value and gradient.  L1 and the feature-image gradient are sums
  over pixels, so a band's share is its own rows.  SSIM's 11x11 window needs 5 rows of each
  neighbouring band: ranks exchange those rows (HaloExchange), each rank's SSIM covers the windows
  centred on its own rows, and the part of its SSIM gradient that falls on a neighbour's rows is sent
  back to that neighbour (BandSSIM).
* Geometry and SH gradients are partial sums over each band's pixels: a reduce-scatter of their flat
  bucket gives every rank the full gradient of its 1/world shard, each rank steps its shard
  (ShardedFlatAdam) and an all-gather returns the stepped parameters to every rank -- on the wire an
  all-reduce.

Collectives are torch.distributed calls (NCCL on GPUs, gloo on CPU), issued in the same order on
every rank.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .parallel import row_bands

HALO = 5  # rows of a neighbouring band the 11x11 SSIM window reaches


def band_reach_mask(means2D: torch.Tensor, radii: torch.Tensor, y0: int, y1: int) -> torch.Tensor:
    """Gaussians that can touch a tile of the rows [y0, y1): visible (radius > 0) and within reach of
    the band's tile rows.  A superset of the gaussians the band bins: the opacity-aware half-height
    k sqrt(Sigma_yy) (k <= sqrt(2 ln 255) < 3.34) is at most 1.12 radius (radius = 3 sqrt(lambda_max)),
    and tile rows round outwards by less than 16 pixels."""
    reach = radii * 1.12 + 1.0
    v = means2D[:, 1]
    return (radii > 0) & (v + reach >= float(y0 - 16)) & (v - reach < float(y1 + 16))


class FeatureShards:
    """The feature table split over the group's ranks: by contiguous row blocks, or by an owner map.

    rows [n_local, C] holds the rows this rank owns, in ascending global id (a leaf: its gradient is
    `rows.grad`, summed over every band by combine()).  dispatch(ids) returns the rows of any sorted
    set of global ids, fetched from their owners; combine(ids, grads) adds per-row gradients into the
    owners' rows.grad.

    starts: optional block boundaries ([world + 1] ints from 0 to n, non-decreasing): rank r owns rows
    [starts[r], starts[r + 1]).  Equal blocks by default; a scene ordered by band_order() passes the
    blocks that make each rank own the rows of its band.

    owner: optional [n] tensor of owning ranks.  Giving each row to the band whose pixels hold its
    gaussian's centre keeps most of a band's rows on its own rank, so that dispatch and combine move
    only the rows of gaussians that reach across a band boundary.  With an owner map, init takes the
    owned global ids (a 1-D int64 tensor) instead of a [start, end) block."""

    def __init__(self, n: int, channels: int, rank: int, world: int, device, group=None, init=None, owner=None,
                 starts=None):
        self.n, self.channels, self.rank, self.world, self.group = n, channels, rank, world, group
        if owner is not None and starts is not None:
            raise ValueError("give an owner map or block boundaries, not both")
        if owner is None:
            self.owner = None
            if starts is None:
                starts = [n * r // world for r in range(world + 1)]
            starts = [int(x) for x in starts]
            if (len(starts) != world + 1 or starts[0] != 0 or starts[-1] != n
                    or any(b < a for a, b in zip(starts, starts[1:]))):
                raise ValueError("starts must rise from 0 to n in world + 1 steps")
            self.starts = starts
            self.start, self.end = self.starts[rank], self.starts[rank + 1]
            local = self.end - self.start
            rows = init(self.start, self.end) if init is not None else torch.zeros(local, channels)
            self._bounds = torch.tensor(self.starts[1:], dtype=torch.int64, device=device)
        else:
            self.owner = owner.to(device=device, dtype=torch.int64)
            if self.owner.shape != (n,) or (n and (int(self.owner.min()) < 0 or int(self.owner.max()) >= world)):
                raise ValueError("owner must hold one rank in [0, world) per row")
            self.ids_local = torch.nonzero(self.owner == rank).squeeze(1)
            self.local_of = torch.full((n,), -1, dtype=torch.int64, device=device)
            self.local_of[self.ids_local] = torch.arange(self.ids_local.numel(), device=device)
            local = self.ids_local.numel()
            rows = init(self.ids_local) if init is not None else torch.zeros(local, channels)
        self.rows = rows.to(device=device, dtype=torch.float32).contiguous().requires_grad_(True)
        self.rows.grad = torch.zeros_like(self.rows)
        self._plan = None
        self._side = None  # stream of dispatch_async

    def _local(self, ids: torch.Tensor) -> torch.Tensor:
        """Positions in rows of owned global ids."""
        return ids - self.start if self.owner is None else self.local_of[ids]

    def dispatch(self, ids: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Rows of the sorted global ids `ids` ([M] int64), in that order ([M, C]; written into `out`
        when given, a contiguous [M, C] tensor)."""
        if self.world == 1:
            self._plan = None
            return self.rows.detach()[self._local(ids)]
        if self.owner is None:
            # Sorted ids and contiguous owners keep every owner's requests in one slice of ids.
            own = torch.searchsorted(self._bounds, ids, right=True)
            perm, grouped = None, ids
        else:
            own = self.owner[ids]
            perm = torch.argsort(own, stable=True)  # requests grouped by owner, ascending within each
            grouped = ids[perm]
        send_counts = torch.bincount(own, minlength=self.world)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        send, recv = send_counts.tolist(), recv_counts.tolist()
        wanted = torch.empty(sum(recv), dtype=ids.dtype, device=ids.device)
        dist.all_to_all_single(wanted, grouped.contiguous(), output_split_sizes=recv, input_split_sizes=send,
                               group=self.group)
        local = self._local(wanted)
        served = self.rows.detach()[local].contiguous()
        if out is not None and perm is None:
            got = out
        else:
            got = torch.empty(ids.numel(), self.channels, dtype=served.dtype, device=served.device)
        dist.all_to_all_single(got, served, output_split_sizes=send, input_split_sizes=recv, group=self.group)
        if perm is not None:
            ordered = out if out is not None else torch.empty_like(got)
            ordered[perm] = got
            got = ordered
        self._plan = (send, recv, local, perm)
        return got

    def dispatch_async(self, ids: torch.Tensor):
        """dispatch(ids) with the fetch queued on a side stream: the counts are exchanged now (a host
        read), then both all-to-alls and the owners' gather run on the side stream while the caller
        queues other work.  Returns a callable that makes the current stream wait for the fetch and
        returns the rows.  CPU tensors, one rank or an owner map: the plain dispatch, done now."""
        if self.world == 1 or not ids.is_cuda or self.owner is not None:
            rows = self.dispatch(ids)
            return lambda: rows
        own = torch.searchsorted(self._bounds, ids, right=True)
        send_counts = torch.bincount(own, minlength=self.world)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        send, recv = send_counts.tolist(), recv_counts.tolist()
        current = torch.cuda.current_stream(ids.device)
        if self._side is None:
            self._side = torch.cuda.Stream(ids.device)
        side = self._side
        side.wait_stream(current)
        with torch.cuda.stream(side):
            wanted = torch.empty(sum(recv), dtype=ids.dtype, device=ids.device)
            dist.all_to_all_single(wanted, ids, output_split_sizes=recv, input_split_sizes=send, group=self.group)
            local = self._local(wanted)
            served = self.rows.detach()[local].contiguous()
            got = torch.empty(ids.numel(), self.channels, dtype=served.dtype, device=ids.device)
            dist.all_to_all_single(got, served, output_split_sizes=send, input_split_sizes=recv, group=self.group)
        ids.record_stream(side)
        self._plan = (send, recv, local, None)

        def finish():
            waiting = torch.cuda.current_stream(ids.device)
            waiting.wait_stream(side)
            got.record_stream(waiting)
            local.record_stream(waiting)
            return got

        return finish

    def combine(self, ids: torch.Tensor, grads: torch.Tensor) -> None:
        """Adds grads ([M, C], rows of the ids of the last dispatch) into the owners' rows.grad."""
        if self.world == 1:
            self.rows.grad.index_add_(0, self._local(ids), grads)
            return
        send, recv, local, perm = self._plan
        outgoing = grads if perm is None else grads[perm]
        back = torch.empty(sum(recv), self.channels, dtype=grads.dtype, device=grads.device)
        dist.all_to_all_single(back, outgoing.contiguous(), output_split_sizes=recv, input_split_sizes=send,
                               group=self.group)
        # Each requester's ids are distinct, so within its slice every row is added once: a gather, an
        # add and a scatter per slice instead of one float atomic per element.
        g, off = self.rows.grad, 0
        for k in recv:
            if k:
                idx = local[off:off + k]
                g[idx] = g[idx] + back[off:off + k]
            off += k


def band_order(means2D: torch.Tensor, radii: torch.Tensor, bands: list[tuple[int, int]]):
    """An order of the scene's gaussians in which rank r's block of rows is the gaussians of its band.

    Each visible gaussian goes to the band whose rows hold its projected centre (clamped into the
    image); the invisible ones fill the ranks with the fewest rows, towards n / world each, so that
    the feature Adam steps stay as even as the bands allow.  Returns (perm [n] int64: the global id
    at each new position, ascending within each block; starts: the block boundaries for
    FeatureShards).  With the scene's rows permuted by perm, in-place band rendering fetches only the
    rows of gaussians whose footprints reach across a band boundary."""
    n, world = means2D.shape[0], len(bands)
    dev = means2D.device
    ends = torch.tensor([b[1] for b in bands[:-1]], dtype=torch.float32, device=dev)
    y = means2D[:, 1].detach().clamp(0.0, float(bands[-1][1] - 1))
    owner = torch.searchsorted(ends, y, right=True).to(torch.int64)
    visible = radii > 0
    counts = torch.bincount(owner[visible], minlength=world).tolist()
    hidden = torch.nonzero(~visible).squeeze(1)
    left = hidden.numel()
    # Water-fill: raise the smallest blocks first.
    share = [0] * world
    for r in sorted(range(world), key=lambda r: counts[r]):
        target = n // world + (1 if r < n % world else 0)
        take = min(left, max(0, target - counts[r]))
        share[r] += take
        left -= take
    for i in range(left):
        share[i % world] += 1
    owner[hidden] = torch.repeat_interleave(torch.arange(world, device=dev), torch.tensor(share, device=dev))
    perm = torch.argsort(owner, stable=True)
    sizes = torch.bincount(owner, minlength=world).tolist()
    starts = [0]
    for k in sizes:
        starts.append(starts[-1] + k)
    return perm, starts


def band_owner(means2D: torch.Tensor, radii: torch.Tensor, bands: list[tuple[int, int]]) -> torch.Tensor:
    """An owner map for FeatureShards: each visible gaussian goes to the band whose rows hold its
    projected centre (clamped into the image), each invisible one to rank id % world."""
    n, world = means2D.shape[0], len(bands)
    ends = torch.tensor([b[1] for b in bands[:-1]], dtype=torch.float32, device=means2D.device)
    y = means2D[:, 1].detach().clamp(0.0, float(bands[-1][1] - 1))
    owner = torch.searchsorted(ends, y, right=True).to(torch.int64)
    spare = torch.arange(n, device=means2D.device) % world
    return torch.where(radii > 0, owner, spare)


class HaloExchange:
    """Neighbouring bands' rows for a band image: extend() returns the band with up to HALO rows of the
    band above and below it (fewer at the image's top and bottom edges); fold() takes a gradient over
    that extended image, sends the halo rows' parts to their owners and adds what the neighbours
    send into the band's own rows.  Every band must have at least HALO rows."""

    def __init__(self, bands: list[tuple[int, int]], rank: int, group=None):
        self.bands, self.rank, self.group = bands, rank, group
        self.world = len(bands)
        y0, y1 = bands[rank]
        if y1 - y0 < HALO and self.world > 1:
            raise ValueError(f"band {rank} has {y1 - y0} rows; the SSIM halo needs at least {HALO}")
        self.top = HALO if rank > 0 else 0
        self.bottom = HALO if rank < self.world - 1 else 0

    def _swap(self, up: torch.Tensor | None, down: torch.Tensor | None, like: torch.Tensor):
        """Sends `up` to the rank above and `down` to the rank below; returns what they send back."""
        ops, from_up, from_down = [], None, None
        shape = (HALO,) + tuple(like.shape[1:])
        if self.rank > 0:
            from_up = torch.empty(shape, dtype=like.dtype, device=like.device)
            ops += [dist.P2POp(dist.isend, up.contiguous(), self.rank - 1, group=self.group),
                    dist.P2POp(dist.irecv, from_up, self.rank - 1, group=self.group)]
        if self.rank < self.world - 1:
            from_down = torch.empty(shape, dtype=like.dtype, device=like.device)
            ops += [dist.P2POp(dist.isend, down.contiguous(), self.rank + 1, group=self.group),
                    dist.P2POp(dist.irecv, from_down, self.rank + 1, group=self.group)]
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        return from_up, from_down

    def extend(self, band: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return band
        above, below = self._swap(band[:HALO], band[-HALO:], band)
        parts = ([above] if above is not None else []) + [band] + ([below] if below is not None else [])
        return torch.cat(parts, dim=0)

    def fold(self, grad_ext: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return grad_ext
        h = grad_ext.shape[0] - self.top - self.bottom
        own = grad_ext[self.top:self.top + h].clone()
        up = grad_ext[:self.top] if self.top else None
        down = grad_ext[self.top + h:] if self.bottom else None
        from_up, from_down = self._swap(up, down, grad_ext)
        if from_up is not None:
            own[:HALO] += from_up
        if from_down is not None:
            own[-HALO:] += from_down
        return own


class BandSSIM(torch.autograd.Function):
    """This band's share of the full image's mean SSIM: the sum of the SSIM map over the band's own
    rows divided by the full image's H * W * 3, computed on the band extended by the halo rows, so
    every window sees the pixels the full image's would.  The backward keeps only the own rows'
    windows (the neighbours' windows are theirs) and folds the halo part of the gradient back.

    ssim_fns = (forward(rendered, gt) -> (map, d_mu, d_aa, d_ab), backward(grad_mean [1], rendered, gt,
    d_mu, d_aa, d_ab) -> grad), the fused SSIM pair, whose backward scales by 1 / (rows * W * 3) of
    the image it is given."""

    @staticmethod
    def forward(ctx, band, gt_ext, halo: HaloExchange, ssim_fns, full_height: int):
        ext = halo.extend(band.contiguous())
        smap, d_mu, d_aa, d_ab = ssim_fns[0](ext, gt_ext)
        h = band.shape[0]
        own = smap[halo.top:halo.top + h]
        ctx.save_for_backward(ext, gt_ext, d_mu, d_aa, d_ab)
        ctx.halo, ctx.fns, ctx.h, ctx.full_height = halo, ssim_fns, h, full_height
        return own.sum(dtype=torch.float64).to(torch.float32) / float(full_height * band.shape[1] * 3)

    @staticmethod
    def backward(ctx, grad):
        ext, gt_ext, d_mu, d_aa, d_ab = ctx.saved_tensors
        halo, h = ctx.halo, ctx.h
        keep = torch.zeros(ext.shape[0], 1, 1, dtype=ext.dtype, device=ext.device)
        keep[halo.top:halo.top + h] = 1.0
        # The kernel divides by the extended image's size; rescale to the full image's.
        grad_mean = (grad.reshape(1) * (ext.shape[0] / ctx.full_height)).to(ext.dtype).contiguous()
        g_ext = ctx.fns[1](grad_mean, ext, gt_ext, d_mu * keep, d_aa * keep, d_ab * keep)
        return halo.fold(g_ext), None, None, None, None


def gpu_ssim_fns():
    """The fused SSIM kernels of this library as BandSSIM's ssim_fns."""
    from .rasterizer import _get_rasterizer

    ext = _get_rasterizer()
    return ext.ssim_forward, ext.ssim_backward


def bin_band(means2D, depths, radii, conics, colors, opacities, width: int, y0: int, y1: int):
    """Bins the band [y0, y1) over the whole scene (no gradient) and compacts it: ids [M] (sorted global
    ids of the gaussians in the band's lists), values [pairs] renamed to positions in ids, ranges, and
    the packed conic / color_opacity rows of ids."""
    from .gaussian_rasterizer import _bin

    with torch.no_grad():
        conic, co, values, ranges, _ = _bin(means2D.contiguous(), depths.contiguous(), radii.contiguous(),
                                            conics.contiguous(), colors.contiguous(), opacities.contiguous(), width,
                                            y1 - y0, origin_y=y0)
        n = means2D.shape[0]
        mask = torch.zeros(n, dtype=torch.bool, device=means2D.device)
        mask[values.long()] = True
        ids = torch.nonzero(mask).squeeze(1)
        rename = torch.empty(n, dtype=torch.int32, device=means2D.device)
        rename[ids] = torch.arange(ids.numel(), dtype=torch.int32, device=means2D.device)
        values_c = rename[values.long()].contiguous()
        return ids, values_c, ranges, conic[ids].contiguous(), co[ids].contiguous()


def band_table(means2D, radii, y0: int, y1: int, start: int, end: int):
    """The table a rank that owns the feature rows [start, end) renders the band [y0, y1) over: rows in
    ascending global id -- the a reachable gaussians below start, the owned block (all of it, in
    place), then the b reachable gaussians from end on.  Returns (pos_ids [a + n_local + b]: the global
    id of each table row, remote_ids [a + b]: the sorted ids of the rows to fetch, a).  The reach is
    band_reach_mask's superset, so a few fetched rows (and unreachable owned rows) hold no pair."""
    with torch.no_grad():
        dev = means2D.device
        reach = band_reach_mask(means2D, radii, y0, y1)
        reach[start:end] = False
        remote_ids = torch.nonzero(reach).squeeze(1)
        a = int(torch.searchsorted(remote_ids, torch.tensor([start], device=dev)).item())
        pos_ids = torch.cat([remote_ids[:a], torch.arange(start, end, device=dev), remote_ids[a:]])
        return pos_ids, remote_ids, a


def bin_table(pos_ids, means2D, depths, radii, conics, colors, opacities, width: int, y0: int, y1: int):
    """Bins the band [y0, y1) over the table rows pos_ids (ascending global ids).  Every per-gaussian
    step of the binning is independent of the others and both sorts are stable in table order, which
    is global-id order, so the lists are the full-scene band's lists with each id replaced by its table
    row.  Returns (values in table rows, ranges, the packed conic / color_opacity rows of the table)."""
    from .gaussian_rasterizer import _bin

    with torch.no_grad():
        def rows(t):
            return t.detach()[pos_ids].contiguous()

        conic, co, values, ranges, _ = _bin(rows(means2D), rows(depths), rows(radii), rows(conics), rows(colors),
                                            rows(opacities), width, y1 - y0, origin_y=y0)
        return values, ranges, conic, co


def bin_band_in_place(means2D, depths, radii, conics, colors, opacities, width: int, y0: int, y1: int, start: int,
                      end: int):
    """bin_band for a rank that owns the feature rows [start, end): band_table, then bin_table.
    Returns (pos_ids, values in table rows, ranges, the packed conic / color_opacity rows of the table,
    remote_ids, a)."""
    pos_ids, remote_ids, a = band_table(means2D, radii, y0, y1, start, end)
    values, ranges, conic, co = bin_table(pos_ids, means2D, depths, radii, conics, colors, opacities, width, y0, y1)
    return pos_ids, values, ranges, conic, co, remote_ids, a


class CompactBandRender(torch.autograd.Function):
    """The fused RGB + feature blend of a band over the compact set of gaussians its lists hold: the
    kernels see exactly the per-entry data and list order of the full-scene call, so the outputs are the
    same bit for bit; the backward runs the fused walk on the compact rows and scatters the geometric
    gradients back to the scene's rows (the feature rows' gradient stays compact, for the owners)."""

    @staticmethod
    def forward(ctx, means2D, conics, colors, opacities, rows, binned, background, width: int, y0: int, y1: int,
                grad_rows=None):
        """grad_rows: when given, the feature rows' gradient is added into it (rows then takes none)."""
        from .gaussian_rasterizer import render_binned_with_features

        ids, values_c, ranges, conic_c, co_c = binned[:5]
        m2c = means2D.detach()[ids].contiguous()
        image, feat, final_T, n_contrib = render_binned_with_features(values_c, ranges, m2c, conic_c, co_c,
                                                                      rows.contiguous(), background, width, y1 - y0,
                                                                      origin_y=y0)
        ctx.save_for_backward(m2c, conic_c, co_c, values_c, ranges, final_T, n_contrib, rows, background, ids)
        ctx.meta = (width, y0, y1, means2D.shape[0])
        ctx.grad_rows = grad_rows
        return image, feat

    @staticmethod
    def backward(ctx, grad_image, grad_feat):
        from .gaussian_rasterizer import rasterize_backward_fused

        m2c, conic_c, co_c, values_c, ranges, final_T, n_contrib, rows, background, ids = ctx.saved_tensors
        width, y0, y1, n = ctx.meta
        if grad_feat is None:
            grad_feat = torch.zeros(y1 - y0, width, rows.shape[1], device=rows.device)
        gm, gc, gcol, go, gf = rasterize_backward_fused(
            grad_image.contiguous() if grad_image is not None else None, background, grad_feat.contiguous(),
            rows.contiguous(), m2c, conic_c, co_c, values_c, ranges, final_T, n_contrib, width, y1 - y0, origin_y=y0,
            grad_features_into=ctx.grad_rows)
        dev = rows.device

        def scatter(g, width_):
            out = torch.zeros(n, width_, device=dev)
            return out.index_add_(0, ids, g)

        g_colors = scatter(gcol, 3) if gcol is not None else torch.zeros(n, 3, device=dev)
        return (scatter(gm, 2), scatter(gc, 3), g_colors, scatter(go, 1), gf, None, None, None, None, None, None)


class PhaseTimer:
    """CUDA events around the phases of a step (when enabled); ms per phase summed over steps."""

    def __init__(self):
        self.enabled = False
        self.marks = []

    def mark(self, name):
        if self.enabled:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.marks.append((name, e))

    def totals(self):
        out = {}
        for (name, a), (_, b) in zip(self.marks, self.marks[1:]):
            if name != "end":
                out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out


class BandSplitTrainer:
    """Training steps of one view split by tile rows over the ranks of `group` (see the module
    docstring).  Holds the replicated geometry + SH leaves with their gradient bucket and Adam, the
    feature shards with theirs, and the band layout; step() runs one forward + backward of the view
    and one optimizer step, and returns the full image's loss (an all-reduce of the bands' shares).

    raw: dict of replicated raw parameters on this rank's device (means, log_scales, quats,
    opacity_logits, sh_dc, sh_rest); features: FeatureShards; lrs: per-parameter learning rates
    (raw's order, then the features')."""

    def __init__(self, raw: dict, features: FeatureShards, camera, lrs: list[float], rank: int, world: int,
                 group=None, row_weights=None):
        from .optim import FlatAdam, ShardedFlatAdam
        from .parallel import GradBucket

        self.raw, self.features, self.camera = raw, features, camera
        self.rank, self.world, self.group = rank, world, group
        self.bands = row_bands(camera.height, world, row_weights)
        self.y0, self.y1 = self.bands[rank]
        self.halo = HaloExchange(self.bands, rank, group)
        self.leaves = list(raw.values())
        # Geometry and SH: with several ranks, each steps 1/world of them (reduce-scatter of the bands'
        # partial gradients, Adam on the shard, all-gather), the same update as an all-reduce and a
        # replicated Adam step with 1/world of the optimizer's memory traffic.
        if world > 1:
            self.opt = ShardedFlatAdam(self.leaves, lrs[:len(self.leaves)], group=group, eps=1e-15)
            self.bucket = self.opt.bucket
        else:
            self.bucket = GradBucket(self.leaves)
            self.opt = FlatAdam(self.leaves, lrs[:len(self.leaves)], eps=1e-15, bucket=self.bucket)
        # With contiguous row blocks each band renders over a table of this rank's own rows (in place,
        # in the optimizer's flat buffer) between the fetched rows of other ranks' gaussians (in its
        # head and tail reserves, in global-id order), and the backward adds straight into the same
        # layout of the gradient bucket.
        self.in_place = world > 1 and features.owner is None
        head = features.start * features.channels if self.in_place else 0
        tail = (features.n - features.end) * features.channels if self.in_place else 0
        self.feature_opt = FlatAdam([features.rows], lrs[len(self.leaves):], eps=1e-15, head=head, tail=tail)
        self.ssim_fns = gpu_ssim_fns()
        self.timer = PhaseTimer()
        self.band_gaussians = 0  # gaussians in this rank's band table (in place) or lists at the last step
        self.fetched_rows = 0  # feature rows fetched from other ranks at the last step

    def geometry_grad(self) -> torch.Tensor:
        """The last step's geometry + SH gradient summed over the bands (flat, the leaves' order).  With
        several ranks this gathers the reduce-scattered shards: a collective every rank must call."""
        if self.world == 1:
            return self.bucket.flat
        shards = torch.empty(self.opt.shard * self.world, device=self.opt.grad_shard.device)
        dist.all_gather_into_tensor(shards, self.opt.grad_shard, group=self.group)
        return shards[:sum(p.numel() for p in self.leaves)]

    def step(self, gt: torch.Tensor, feature_grad: torch.Tensor) -> torch.Tensor:
        """One forward + backward of the view and one optimizer step.  gt: the full view's [H, W, 3]
        float ground truth (on this device; each rank reads its band and halo rows); feature_grad: the
        fixed gradient of this band's [y1 - y0, W, C] feature image (the harness scope).  Returns the
        full image's loss as a device scalar (summed over the ranks)."""
        from .projection import project_gaussians_raw
        from .rasterizer import accumulate_leaf_grads, rasterize
        from .sh import view_colors

        cam, L, t = self.camera, self.raw, self.timer
        H, W = cam.height, cam.width
        y0, y1 = self.y0, self.y1
        t.mark("clear")
        self.bucket.zero_async()
        if not self.in_place:
            self.feature_opt.bucket.zero()
        pose = cam.world_to_camera
        center = -(pose[:3, :3].T @ pose[:3, 3])
        bg = torch.zeros(3, device=pose.device)
        t.mark("project_sh")
        with accumulate_leaf_grads():
            means2D, depths, radii, conics, opacities = project_gaussians_raw(
                L["means"], L["log_scales"], L["quats"], L["opacity_logits"], pose, cam.fx, cam.fy, cam.cx, cam.cy, W,
                H)
            colors = view_colors(L["sh_dc"], L["sh_rest"], L["means"], center, 3, radii)
            if self.world == 1:
                # One band is the whole view: the plain fused path, the shard is the whole table.
                t.mark("render")
                image, feat = rasterize(means2D, depths, radii, conics, colors, opacities, W, H, bg,
                                        self.features.rows)
                ids = None
            elif self.in_place:
                t.mark("bin")
                f = self.features
                pos_ids, remote, a = band_table(means2D, radii, y0, y1, f.start, f.end)
                # The fetch needs only the table: it runs on a side stream while the band is binned.
                pending = f.dispatch_async(remote)
                binned = (pos_ids,) + bin_table(pos_ids, means2D, depths, radii, conics, colors, opacities, W, y0, y1)
                self.band_gaussians = pos_ids.numel()
                self.fetched_rows = remote.numel()
                n_local, Cf = f.end - f.start, f.channels
                # The table: a fetched rows, the owned block (in place), the other fetched rows -- a
                # window of the optimizer's flat buffer around its parameters, and of its bucket.
                lo, hi = (self.feature_opt.head // Cf - a) * Cf, (self.feature_opt.head // Cf + n_local +
                                                                   remote.numel() - a) * Cf
                table = self.feature_opt.flat[lo:hi].view(-1, Cf)
                # Only the rows this step uses are cleared: the owned rows (every one is stepped) and
                # the fetched ones; the rest of the reserve is never read.
                grad_table = self.feature_opt.bucket.flat[lo:hi].view(-1, Cf)
                grad_table.zero_()
                self.feature_opt.bucket.attach()
                t.mark("dispatch")
                fetched = pending()
                table[:a] = fetched[:a]
                table[a + n_local:] = fetched[a:]
                t.mark("render")
                image, feat = CompactBandRender.apply(means2D, conics, colors, opacities, table, binned, bg, W, y0,
                                                      y1, grad_table)
                ids = remote
            else:
                t.mark("bin")
                binned = bin_band(means2D, depths, radii, conics, colors, opacities, W, y0, y1)
                ids = binned[0]
                self.band_gaussians = ids.numel()
                t.mark("dispatch")
                rows = self.features.dispatch(ids).requires_grad_(True)
                t.mark("render")
                image, feat = CompactBandRender.apply(means2D, conics, colors, opacities, rows, binned, bg, W, y0,
                                                      y1)
        t.mark("loss")
        e0, e1 = y0 - self.halo.top, y1 + self.halo.bottom
        # 0.8 L1 + 0.2 (1 - SSIM), the training loop's loss (main.py:179-182), as this band's share.
        l1_share = (image - gt[y0:y1]).abs().sum(dtype=torch.float64).to(torch.float32) / float(H * W * 3)
        ssim_share = BandSSIM.apply(image, gt[e0:e1].contiguous(), self.halo, self.ssim_fns, H)
        loss = 0.8 * l1_share + 0.2 * ((y1 - y0) / H - ssim_share)
        self.bucket.ready()
        t.mark("backward")
        torch.autograd.backward([loss, feat], [None, feature_grad.contiguous()])
        # Feature gradients back to their owners; geometry and SH summed over the bands.
        if self.world > 1:
            t.mark("combine")
            if self.in_place:
                n_local = self.features.end - self.features.start
                self.features.combine(ids, torch.cat([grad_table[:a], grad_table[a + n_local:]]))
            else:
                self.features.combine(ids, rows.grad)
        t.mark("adam")
        self.opt.step()
        self.feature_opt.step()
        total = loss.detach().reshape(1)
        if self.world > 1:
            dist.all_reduce(total, group=self.group)
        t.mark("end")
        return total

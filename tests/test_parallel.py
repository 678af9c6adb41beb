"""Host logic of the multi-GPU paths, on CPU: view sharding, tile-row bands (checked by rendering
bands with the oracle and comparing with the full render), and the flat gradient bucket summed
over two gloo ranks."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from helpers import assert_close_abs, assert_grads_close
from hds_b200 import parallel
from scenes_np import reference_scene


def test_shard_views_cover_every_view_once():
    for world in (1, 2, 3, 8):
        got = sorted(v for r in range(world) for v in parallel.shard_views(64, r, world))
        assert got == list(range(64))


@pytest.mark.parametrize("height, world", [(546, 2), (546, 4), (1080, 8), (17, 2), (48, 3)])
def test_row_bands_partition_whole_tile_rows(height, world):
    rows = (height + 15) // 16
    rng = np.random.default_rng(height)
    for weights in (None, list(rng.random(rows) * 10 + 1)):
        bands = parallel.row_bands(height, world, weights)
        assert len(bands) == world and bands[0][0] == 0 and bands[-1][1] == height
        for (a0, a1), (b0, b1) in zip(bands, bands[1:]):
            assert a1 == b0
        for y0, y1 in bands:
            assert y0 % 16 == 0 and y1 > y0


def test_row_bands_reject_more_bands_than_tile_rows():
    """A 2-tile-row view across 4 ranks would leave two ranks without rows: refused up front."""
    with pytest.raises(ValueError):
        parallel.row_bands(32, 4)
    with pytest.raises(ValueError):
        parallel.row_bands(17, 0)
    assert parallel.row_bands(32, 2) == [(0, 16), (16, 32)]


def test_bucket_zero_async_on_cpu_is_zero():
    params = [torch.randn(10, 3, requires_grad=True), torch.randn(4, requires_grad=True)]
    bucket = parallel.GradBucket(params)
    bucket.flat.fill_(3.0)
    bucket.zero_async()
    bucket.ready()
    assert all(p.grad is v for p, v in zip(params, bucket.views))
    assert torch.count_nonzero(bucket.flat) == 0


def test_flat_adam_reserves_lay_out_around_the_parameters_on_cpu():
    """FlatAdam(head=, tail=): the parameters become views of the flat buffer after `head` zeros, the
    gradient bucket puts their slices at the same offsets, and both buffers end with `tail` zeros
    (the layout only; the step runs the CUDA kernel and is checked on the GPU)."""
    from hds_b200.optim import FlatAdam

    params = [torch.randn(6, 4, requires_grad=True), torch.randn(5, requires_grad=True)]
    values = [p.detach().clone() for p in params]
    head, tail = 12, 20
    opt = FlatAdam(params, [0.1, 0.2], head=head, tail=tail)
    n = 6 * 4 + 5
    assert opt.n == n and opt.head == head and opt.flat.numel() == head + n + tail
    assert torch.count_nonzero(opt.flat[:head]) == 0 and torch.count_nonzero(opt.flat[head + n:]) == 0
    assert torch.equal(opt.flat[head:head + 24].view(6, 4), values[0]) and torch.equal(opt.flat[head + 24:head + n],
                                                                                         values[1])
    assert params[0].data_ptr() == opt.flat[head:].data_ptr()
    opt.zero_grad()
    assert opt.bucket.flat.numel() == head + n + tail
    assert params[0].grad.data_ptr() == opt.bucket.flat[head:].data_ptr()
    assert params[1].grad.data_ptr() == opt.bucket.flat[head + 24:].data_ptr()
    with pytest.raises(ValueError):
        FlatAdam([torch.randn(3, requires_grad=True)], [0.1], head=4, bucket=parallel.GradBucket(params))


def band_render_np(inputs, width, y0, y1, background, features=None):
    """Rows [y0, y1) of the full render: the band is an image of its own whose row 0 lies at row y0
    of the full view (origin_y), with the means in full-image pixels."""
    m2, dep, rad, con, col, opac = inputs
    return oracle.rasterize(m2, dep, rad, con, col, opac, width, y1 - y0, background=background, features=features,
                            origin_y=y0)


def test_bands_stitch_into_the_full_render():
    """Pixel centres and tile rectangles in full-image coordinates make every band's outputs equal
    its rows of the full render bit for bit, features included."""
    width, height = 96, 80
    inputs = reference_scene(5, 3000, width, height)
    feats = np.random.default_rng(2).standard_normal((3000, 8)).astype(np.float32)
    bg = np.array([0.3, 0.5, 0.7], np.float32)
    full = oracle.rasterize(*inputs, width, height, background=bg, features=feats)
    for world in (2, 3, 5):
        parts = [band_render_np(inputs, width, y0, y1, bg, feats) for y0, y1 in parallel.row_bands(height, world)]
        for key in ("image", "final_T", "n_contrib", "features"):
            assert np.array_equal(np.concatenate([p[key] for p in parts], axis=0), full[key]), key


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # 1. The flat bucket sums every parameter's gradient over ranks with one collective.
        params = [torch.zeros(5, 3, requires_grad=True), torch.zeros(7, requires_grad=True)]
        bucket = parallel.GradBucket(params)
        bucket.zero()
        ((params[0] * (rank + 1)).sum() + (params[1] * 10 * (rank + 1)).sum()).backward()
        bucket.all_reduce()
        total = sum(r + 1 for r in range(world))
        ok_bucket = torch.equal(params[0].grad, torch.full((5, 3), float(total))) and \
            torch.equal(params[1].grad, torch.full((7,), 10.0 * total))

        # 2. Tile-row split: each rank renders and back-propagates its band with the oracle; the
        #    all-gathered images and the all-reduced gradients must match the full render.
        width, height = 64, 48
        inputs = reference_scene(9, 1500, width, height)
        m2, dep, rad, con, col, opac = inputs
        y0, y1 = parallel.row_bands(height, world)[rank]
        band = band_render_np(inputs, width, y0, y1, None)
        grad_image = np.random.default_rng(3).random((height, width, 3), dtype=np.float32)
        g = oracle.render_backward(band["ranges"], band["values"], m2, con, col, opac, width, y1 - y0,
                                   band["final_T"], band["n_contrib"], grad_image=grad_image[y0:y1], origin_y=y0)
        grads = [torch.from_numpy(np.ascontiguousarray(x)) for x in g[:4]]
        for t in grads:
            dist.all_reduce(t)
        images = [None] * world
        dist.all_gather_object(images, band["image"])
        out[rank] = {"bucket": ok_bucket, "image": np.concatenate(images, axis=0),
                     "grads": [t.numpy() for t in grads]}
    finally:
        dist.destroy_process_group()


def _gloo_entry(rank, world, port, queue):
    out = {}
    _gloo_worker(rank, world, port, out)
    queue.put((rank, out[rank]))


def test_two_gloo_ranks_bucket_and_band_split():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_gloo_entry, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    width, height = 64, 48
    inputs = reference_scene(9, 1500, width, height)
    m2, dep, rad, con, col, opac = inputs
    full = oracle.rasterize(*inputs, width, height)
    grad_image = np.random.default_rng(3).random((height, width, 3), dtype=np.float32)
    want = oracle.render_backward(full["ranges"], full["values"], m2, con, col, opac, width, height, full["final_T"],
                                  full["n_contrib"], grad_image=grad_image)
    for rank in range(world):
        r = results[rank]
        assert r["bucket"]
        assert np.array_equal(r["image"], full["image"]), "stitched bands differ from the full render"
        for name, got, w in zip(("means2D", "conics", "colors", "opacities"), r["grads"], want[:4]):
            assert_grads_close(got, w, name)


def _adam_reference(params, exp_avg, exp_avg_sq, grads, segment_ends, segment_lrs, step, betas=(0.9, 0.999),
                    eps=1e-15):
    """The Adam element update of hds_adam_step in torch (CPU stand-in for the kernel in the host-logic
    test below; the kernel itself is checked against torch.optim.Adam on the GPU)."""
    b1, b2 = betas
    start = 0
    for end, lr in zip(segment_ends, segment_lrs):
        sl = slice(start, int(end))
        g = grads[sl]
        exp_avg[sl] += (1.0 - b1) * (g - exp_avg[sl])
        exp_avg_sq[sl] = b2 * exp_avg_sq[sl] + (1.0 - b2) * g * g
        step_size = lr / (1.0 - b1 ** step)
        params[sl] -= step_size * exp_avg[sl] / (exp_avg_sq[sl].sqrt() / (1.0 - b2 ** step) ** 0.5 + eps)
        start = int(end)


def _sharded_adam_worker(rank, world, port, queue):
    import torch.distributed as dist

    from hds_b200 import optim

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        optim.adam_step = _adam_reference  # the kernel needs a GPU; the host logic is under test
        gen = torch.Generator().manual_seed(5)
        shapes = [(1001, 3), (77,), (513, 16)]
        params = [torch.randn(s, generator=gen).requires_grad_(True) for s in shapes]
        opt = optim.ShardedFlatAdam(params, [1e-3, 2e-2, 5e-4], group=None)
        grads_seen = []
        for step in range(3):
            opt.zero_grad()
            for p in params:
                g = torch.randn(p.shape, generator=torch.Generator().manual_seed(100 * step + rank + 7))
                p.grad.add_(g)
            grads_seen.append(torch.cat([p.grad.reshape(-1).clone() for p in params]))
            opt.step()
        queue.put((rank, [p.detach().clone() for p in params], grads_seen, opt.shard, opt.world))
    finally:
        dist.destroy_process_group()


def test_sharded_adam_over_two_gloo_ranks_equals_adam_on_summed_gradients():
    """Reduce-scatter, per-rank Adam over its shard and all-gather give every rank the parameters of
    one Adam step on the all-reduced gradients, three steps in a row (segments crossing shard
    boundaries, padding at the end)."""
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_sharded_adam_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {r: (ps, gs, shard, w) for r, ps, gs, shard, w in (queue.get(timeout=240) for _ in range(world))}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0][2] % 64 == 0 and results[0][2] * world >= 1001 * 3 + 77 + 513 * 16
    gen = torch.Generator().manual_seed(5)
    shapes = [(1001, 3), (77,), (513, 16)]
    ref = torch.cat([torch.randn(s, generator=gen).reshape(-1) for s in shapes])
    m, v = torch.zeros_like(ref), torch.zeros_like(ref)
    ends = list(np.cumsum([int(np.prod(s)) for s in shapes]))
    for step in range(3):
        g = results[0][1][step] + results[1][1][step]
        _adam_reference(ref, m, v, g, ends, [1e-3, 2e-2, 5e-4], step + 1)
    for r in range(world):
        got = torch.cat([p.reshape(-1) for p in results[r][0]])
        assert torch.equal(got, ref), f"rank {r}: max diff {float((got - ref).abs().max())}"

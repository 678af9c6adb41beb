"""The tile-row split's exchange logic on CPU, over three gloo ranks (hds_b200.band_split):

* FeatureShards: rows dispatched from their owners equal the full table's rows; gradients combined
  from every band land summed on the owners -- with contiguous row blocks, and with an owner map
  (band_owner on a scene's projected centres), and with uneven blocks of a scene put in band order
  (band_order).
* band_table: the rows a band renders over, in global order around the owned block.
* HaloExchange + BandSSIM (with the oracle's SSIM): the bands' shares add up to the full image's mean
  SSIM, and the folded band gradients equal the full image's SSIM gradient row for row.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from helpers import assert_grads_close

WORLD = 3
N, C = 1000, 8
H, W = 80, 48


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def table_rows(start, end):
    g = torch.arange(start, end, dtype=torch.float32)[:, None]
    return g * C + torch.arange(C, dtype=torch.float32)[None, :]


def rank_ids(rank):
    rng = np.random.default_rng(rank)
    return torch.from_numpy(np.unique(rng.integers(0, N, 300))).long()


def oracle_ssim_fns():
    def fwd(a, b):
        return tuple(torch.from_numpy(x) for x in oracle.ssim_forward(a.detach().numpy(), b.numpy()))

    def bwd(grad_mean, a, b, d_mu, d_aa, d_ab):
        return torch.from_numpy(oracle.ssim_backward(float(grad_mean[0]), a.detach().numpy(), b.numpy(),
                                                     d_mu.numpy(), d_aa.numpy(), d_ab.numpy()))

    return fwd, bwd


def images():
    rng = np.random.default_rng(9)
    gt = rng.random((H, W, 3), dtype=np.float32)
    img = np.clip(gt + 0.2 * rng.standard_normal((H, W, 3)).astype(np.float32), 0, 1).astype(np.float32)
    return img, gt


def _worker(rank, port, queue):
    import torch.distributed as dist

    from hds_b200 import band_split, parallel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        shards = band_split.FeatureShards(N, C, rank, WORLD, "cpu", init=table_rows)
        ids = rank_ids(rank)
        rows = shards.dispatch(ids)
        rows_ok = torch.equal(rows, table_rows(0, N)[ids])
        shards.combine(ids, torch.full((len(ids), C), float(rank + 1)))
        grads = [None] * WORLD
        dist.all_gather_object(grads, (shards.start, shards.rows.grad.numpy().copy()))

        # The same through an owner map: each row owned by the band that holds its centre.
        gen = torch.Generator().manual_seed(4)
        means2D = torch.rand(N, 2, generator=gen) * torch.tensor([float(W), float(H)])
        radii = (torch.rand(N, generator=gen) > 0.1).float() * 3.0
        owner = band_split.band_owner(means2D, radii, parallel.row_bands(H, WORLD))
        mapped = band_split.FeatureShards(N, C, rank, WORLD, "cpu", init=lambda g: table_rows(0, N)[g], owner=owner)
        rows_m = mapped.dispatch(ids)
        mapped_ok = torch.equal(rows_m, table_rows(0, N)[ids])
        mapped.combine(ids, torch.full((len(ids), C), float(rank + 1)))
        grads_m = [None] * WORLD
        dist.all_gather_object(grads_m, (mapped.ids_local.numpy().copy(), mapped.rows.grad.numpy().copy()))

        # The scene in band order: uneven blocks, rank r's block holding the gaussians of band r.
        perm, starts = band_split.band_order(means2D, radii, parallel.row_bands(H, WORLD))
        ordered = band_split.FeatureShards(N, C, rank, WORLD, "cpu", init=lambda a, b: table_rows(0, N)[perm[a:b]],
                                           starts=starts)
        rows_o = ordered.dispatch(ids)
        ordered_ok = torch.equal(rows_o, table_rows(0, N)[perm[ids]])
        ordered.combine(ids, torch.full((len(ids), C), float(rank + 1)))
        grads_o = [None] * WORLD
        dist.all_gather_object(grads_o, (ordered.start, ordered.rows.grad.numpy().copy()))

        img, gt = images()
        bands = parallel.row_bands(H, WORLD)
        y0, y1 = bands[rank]
        halo = band_split.HaloExchange(bands, rank)
        band = torch.from_numpy(img[y0:y1].copy()).requires_grad_(True)
        gt_ext = torch.from_numpy(gt[y0 - halo.top:y1 + halo.bottom].copy())
        share = band_split.BandSSIM.apply(band, gt_ext, halo, oracle_ssim_fns(), H)
        share.backward()
        shares = [None] * WORLD
        dist.all_gather_object(shares, (float(share), band.grad.numpy().copy()))
        queue.put((rank, {"rows_ok": rows_ok, "grads": grads, "ssim": shares, "mapped_ok": mapped_ok,
                          "grads_mapped": grads_m, "owner": owner.numpy(), "ordered_ok": ordered_ok,
                          "grads_ordered": grads_o, "starts": starts}))
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def results():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, queue)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = dict(queue.get(timeout=240) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


def test_feature_shards_dispatch_and_combine(results):
    assert all(results[r]["rows_ok"] for r in range(WORLD))
    want = np.zeros((N, C), np.float32)
    for r in range(WORLD):
        want[rank_ids(r).numpy()] += r + 1
    got = np.zeros((N, C), np.float32)
    for start, g in results[0]["grads"]:
        got[start:start + len(g)] = g
    assert np.array_equal(got, want)


def test_feature_shards_with_an_owner_map(results):
    assert all(results[r]["mapped_ok"] for r in range(WORLD))
    want = np.zeros((N, C), np.float32)
    for r in range(WORLD):
        want[rank_ids(r).numpy()] += r + 1
    got = np.full((N, C), np.nan, np.float32)
    owner = results[0]["owner"]
    for r, (ids_local, g) in enumerate(results[0]["grads_mapped"]):
        assert np.array_equal(owner[ids_local], np.full(len(ids_local), r))
        got[ids_local] = g
    assert np.array_equal(got, want)  # every row owned exactly once, gradients summed


def test_feature_shards_in_band_order(results):
    assert all(results[r]["ordered_ok"] for r in range(WORLD))
    want = np.zeros((N, C), np.float32)
    for r in range(WORLD):
        want[rank_ids(r).numpy()] += r + 1
    got = np.full((N, C), np.nan, np.float32)
    starts = results[0]["starts"]
    for r, (start, g) in enumerate(results[0]["grads_ordered"]):
        assert start == starts[r] and len(g) == starts[r + 1] - starts[r]
        got[start:start + len(g)] = g
    assert np.array_equal(got, want)


def test_band_order_puts_each_band_in_its_block():
    from hds_b200 import band_split, parallel

    gen = torch.Generator().manual_seed(5)
    n, world = 2000, 3
    means2D = torch.rand(n, 2, generator=gen) * torch.tensor([float(W), 1.5 * H]) - torch.tensor([0.0, 0.25 * H])
    radii = (torch.rand(n, generator=gen) > 0.3).float() * 3.0
    bands = parallel.row_bands(H, world, [1.0 + 4.0 * (y < H // 4) for y in range((H + 15) // 16)])
    perm, starts = band_split.band_order(means2D, radii, bands)
    assert sorted(perm.tolist()) == list(range(n)) and starts[0] == 0 and starts[-1] == n
    y = means2D[:, 1].clamp(0.0, H - 1.0)
    for r, (y0, y1) in enumerate(bands):
        block = perm[starts[r]:starts[r + 1]]
        assert torch.all(block[1:] > block[:-1])  # ascending within a block
        vis = block[radii[block] > 0]
        lo = y0 if r > 0 else -1.0
        assert torch.all((y[vis] >= lo) & (y[vis] < y1)), r
        # Every visible gaussian of band r is in block r.
        in_band = torch.nonzero((radii > 0) & (y >= lo) & (y < y1)).squeeze(1)
        assert set(in_band.tolist()) <= set(block.tolist())
    # The hidden gaussians raise the smaller blocks towards n / world before the larger ones grow.
    sizes = [starts[r + 1] - starts[r] for r in range(world)]
    vis_sizes = [int(((radii > 0) & (y >= (bands[r][0] if r else -1.0)) & (y < bands[r][1])).sum())
                 for r in range(world)]
    assert sum(sizes) == n and all(s >= v for s, v in zip(sizes, vis_sizes))
    assert max(sizes) == max(max(vis_sizes), -(-n // world))


def test_band_ssim_matches_full_image(results):
    img, gt = images()
    smap, d_mu, d_aa, d_ab = oracle.ssim_forward(img, gt)
    full_grad = oracle.ssim_backward(1.0, img, gt, d_mu, d_aa, d_ab)
    shares = results[0]["ssim"]
    total = sum(s for s, _ in shares)
    np.testing.assert_allclose(total, smap.astype(np.float64).mean(), rtol=1e-6)
    stitched = np.concatenate([g for _, g in shares], axis=0)
    assert_grads_close(stitched, full_grad, "SSIM gradient stitched from bands")


def test_band_table_is_in_global_order_around_the_owned_block():
    """band_table (the rows a rank renders its band over): ascending global ids, the whole owned block
    in place after the a reachable ids below it, and exactly the reachable ids outside the block as
    the rows to fetch."""
    from hds_b200 import band_split

    gen = torch.Generator().manual_seed(8)
    n = 3000
    means2D = torch.rand(n, 2, generator=gen) * torch.tensor([float(W), 2.0 * H]) - torch.tensor([0.0, 0.5 * H])
    radii = (torch.rand(n, generator=gen) > 0.2).float() * (1.0 + 6.0 * torch.rand(n, generator=gen))
    y0, y1, start, end = 32, 64, 1100, 2100
    pos_ids, remote, a = band_split.band_table(means2D, radii, y0, y1, start, end)
    reach = band_split.band_reach_mask(means2D, radii, y0, y1)
    want_remote = torch.tensor([i for i in range(n) if bool(reach[i]) and not start <= i < end], dtype=torch.int64)
    assert torch.equal(remote, want_remote)
    assert a == int((want_remote < start).sum())
    assert torch.all(pos_ids[1:] > pos_ids[:-1])
    assert torch.equal(pos_ids[a:a + end - start], torch.arange(start, end))
    assert pos_ids.numel() == remote.numel() + end - start

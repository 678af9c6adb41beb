"""The tile-row split end to end on two GPUs (hds_b200.band_split over NCCL): one training step of a
config-4-like view split into two bands gives the same loss and the same gradients -- geometry and SH
after their all-reduce, features after the combine at their owners -- as the whole view on one GPU,
with the feature table split in row blocks, by an owner map, or in uneven blocks of a scene put in
band order (both runs then render the same reordered scene).  Needs two GPUs; skipped otherwise."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

N, C = 60_000, 32


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, port, queue, mode="blocks"):
    import torch.distributed as dist

    from hds_b200 import band_split, optim, scenes

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device)
    try:
        s = scenes.config4(1, channels=0, n=N)
        cam = s.cameras[0].to(device)
        op = s.opacities.clamp(1e-6, 1 - 1e-6)
        raw = {"means": s.means, "log_scales": torch.log(s.scales), "quats": s.quats,
               "opacity_logits": torch.log(op / (1 - op)), "sh_dc": s.sh_dc, "sh_rest": s.sh_rest}
        raw = {k: v.to(device).contiguous().requires_grad_(True) for k, v in raw.items()}
        table = torch.randn(N, C, generator=torch.Generator().manual_seed(3))
        starts = None
        if mode == "band_order":
            from hds_b200.parallel import row_bands
            from hds_b200.projection import project_gaussians_raw

            with torch.no_grad():
                m2, _, rad, _, _ = project_gaussians_raw(raw["means"], raw["log_scales"], raw["quats"],
                                                         raw["opacity_logits"], cam.world_to_camera, cam.fx, cam.fy,
                                                         cam.cx, cam.cy, cam.width, cam.height)
            perm, two_starts = band_split.band_order(m2, rad, row_bands(cam.height, 2))
            raw = {k: v.detach()[perm].contiguous().requires_grad_(True) for k, v in raw.items()}
            table = table[perm.cpu()]
            starts = two_starts if world > 1 else None
        if mode == "owner_map" and world > 1:
            owner = torch.randint(0, world, (N,), generator=torch.Generator().manual_seed(6))
            feats = band_split.FeatureShards(N, C, rank, world, device, init=lambda ids: table[ids.cpu()].clone(),
                                             owner=owner)
            ids_local = feats.ids_local.cpu().numpy()
        else:
            feats = band_split.FeatureShards(N, C, rank, world, device, init=lambda a, b: table[a:b].clone(),
                                             starts=starts)
            ids_local = np.arange(feats.start, feats.end)
        lrs = [optim.REFERENCE_LRS[k] for k in raw] + [optim.REFERENCE_LRS["features"]]
        trainer = band_split.BandSplitTrainer(raw, feats, cam, lrs, rank, world)
        H, W = cam.height, cam.width
        gt = torch.rand(H, W, 3, generator=torch.Generator().manual_seed(4)).to(device)
        fgrad = torch.rand(H, W, C, generator=torch.Generator().manual_seed(5)).to(device) / (H * W)
        loss = trainer.step(gt, fgrad[trainer.y0:trainer.y1])
        out = {"loss": float(loss), "geometry": trainer.geometry_grad().cpu().numpy(),
               "features": (ids_local, feats.rows.grad.cpu().numpy()), "bands": trainer.bands,
               "fetched": trainer.fetched_rows}
        queue.put((rank, out))
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


def _launch(world, mode="blocks"):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, queue, mode)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(queue.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return out


@pytest.mark.parametrize("mode", ["blocks", "owner_map", "band_order"])
def test_two_band_step_matches_one_gpu(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("the tile-row split test needs two GPUs")
    from helpers import assert_grads_close

    one = _launch(1, mode)[0]
    two = _launch(2, mode)
    assert len(two[0]["bands"]) == 2
    np.testing.assert_allclose(two[0]["loss"], one["loss"], rtol=1e-5)
    assert two[0]["loss"] == two[1]["loss"]
    assert np.array_equal(two[0]["geometry"], two[1]["geometry"]), "ranks disagree after the all-reduce"
    off = 0
    for name, width in (("means", 3), ("log_scales", 3), ("quats", 4), ("opacity_logits", 1), ("sh_dc", 3),
                        ("sh_rest", 45)):
        seg = slice(off, off + N * width)
        assert_grads_close(two[0]["geometry"][seg], one["geometry"][seg], f"{name} gradients, 2 bands vs 1 GPU")
        off += N * width
    assert off == len(one["geometry"])
    got = np.full((N, C), np.nan, np.float32)
    for r in range(2):
        ids_local, g = two[r]["features"]
        got[ids_local] = g
    assert_grads_close(got, one["features"][1], "feature gradients, 2 bands vs 1 GPU")
    if mode == "band_order":
        # Only gaussians reaching across the band edge are fetched.
        assert two[0]["fetched"] + two[1]["fetched"] < N // 10

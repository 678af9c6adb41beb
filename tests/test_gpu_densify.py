"""Densification on the device against the reference's own densify_and_prune
(tests/golden/densify.npz, written by tests/golden/make_golden.py from utils/gaussian.py on CPU, with
its torch.normal draws recorded): the same population (rows, order and count) after clone, split and
prune, the same parameters (copies bit for bit; split children's means and log-scales within float
rounding of the reference's torch arithmetic) and the same Adam moments (copied for surviving rows,
zero for appended ones).  Also the statistics kernel against add_densification_stats."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REF = ("means", "scales", "quats", "opacities", "sh_dc", "sh_rest")  # the reference's names, in our order


def _opt_from_fixture(g):
    from hds_b200.optim import FlatAdam

    leaves = [torch.from_numpy(g[f"in_param_{k}"]).cuda().requires_grad_(True) for k in REF]
    opt = FlatAdam(leaves, [1e-3] * len(leaves))
    off = 0
    for k, p in zip(REF, opt.params):
        n = p.numel()
        opt.exp_avg[off:off + n] = torch.from_numpy(g[f"in_m_{k}"].reshape(-1)).cuda()
        opt.exp_avg_sq[off:off + n] = torch.from_numpy(g[f"in_v_{k}"].reshape(-1)).cuda()
        off += n
    return opt


def test_densify_and_prune_matches_the_reference(golden):
    from hds_b200.densify import DensifyStats, densify_and_prune

    g = golden("densify.npz")
    opt = _opt_from_fixture(g)
    n = g["in_param_means"].shape[0]
    stats = DensifyStats(n, "cuda")
    stats.grad_accum.copy_(torch.from_numpy(g["in_grad_accum"]))
    stats.denom.copy_(torch.from_numpy(g["in_denom"]))
    stats.max_radii2D.copy_(torch.from_numpy(g["in_max_radii2D"]))
    new_opt, new_stats = densify_and_prune(opt, stats, grad_threshold=0.0002, percent_dense=0.01, min_opacity=0.005,
                                           extent=float(g["extent"]), max_screen_size=20,
                                           normals=torch.from_numpy(g["normals"]).cuda())
    n_new = g["out_param_means"].shape[0]
    assert new_opt.params[0].shape[0] == n_new and n_new != n
    for k, p in zip(REF, new_opt.params):
        got, want = p.detach().cpu().numpy(), g[f"out_param_{k}"]
        assert got.shape == want.shape, k
        if k in ("means", "scales"):
            np.testing.assert_allclose(got, want, rtol=2e-6, atol=2e-7, err_msg=k)
        else:
            assert np.array_equal(got, want), f"{k} differs"
    off = 0
    for k, p in zip(REF, new_opt.params):
        m = p.numel()
        assert np.array_equal(new_opt.exp_avg[off:off + m].cpu().numpy(), g[f"out_m_{k}"].reshape(-1)), f"exp_avg {k}"
        assert np.array_equal(new_opt.exp_avg_sq[off:off + m].cpu().numpy(), g[f"out_v_{k}"].reshape(-1)), k
        off += m
    assert float(new_stats.denom.abs().sum()) == 0.0 and new_stats.denom.shape == (n_new, 1)


def test_densify_stats_match_the_reference_formula():
    from hds_b200.densify import DensifyStats

    gen = torch.Generator().manual_seed(2)
    n, W, H = 5000, 979, 546
    stats = DensifyStats(n, "cuda")
    want_max = torch.zeros(n)
    want_acc = torch.zeros(n, 1)
    want_den = torch.zeros(n, 1)
    for _ in range(3):
        grad = torch.randn(n, 2, generator=gen) * 1e-3
        radii = torch.rand(n, generator=gen) * 10.0
        radii[torch.rand(n, generator=gen) < 0.3] = 0.0
        stats.add(grad.cuda(), radii.cuda(), W, H)
        vis = radii > 0
        want_max = torch.where(vis, torch.maximum(want_max, radii), want_max)
        scale = torch.tensor([0.5 * W, 0.5 * H])
        want_acc[vis] += (grad * scale)[vis].norm(dim=-1, keepdim=True)
        want_den[vis] += 1
    assert torch.equal(stats.max_radii2D.cpu(), want_max)
    assert torch.equal(stats.denom.cpu(), want_den)
    np.testing.assert_allclose(stats.grad_accum.cpu().numpy(), want_acc.numpy(), rtol=1e-6, atol=1e-9)

"""The projection's analytic backward (projection.cu:114-197 of the reference, restated in the oracle
and bit-identical on the GPU) against autograd of an fp64 torch restatement of its forward
(projection.cu:36-111).  The reference has no CPU projection, so this pins the gradients to the
derivative of the forward itself, including the field-of-view clamp and the near-plane cases."""
import numpy as np
import torch

import oracle
from hds_b200 import scenes


def quat_to_rotmat(q):
    w, x, y, z = q.unbind(-1)
    return torch.stack([
        1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
        2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
        2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1).reshape(-1, 3, 3)


def project_torch(means, scales, quats, w2c, fx, fy, cx, cy, width, height, near=0.2, low_pass=0.3, fov=1.3):
    R, t = w2c[:3, :3], w2c[:3, 3]
    p = means @ R.T + t
    z = torch.clamp(p[:, 2], min=near)
    z_inv = 1.0 / (z + 1e-6)
    lim_x, lim_y = fov * (0.5 * width / fx), fov * (0.5 * height / fy)
    jx = torch.clamp(p[:, 0] * z_inv, -lim_x, lim_x) * z
    jy = torch.clamp(p[:, 1] * z_inv, -lim_y, lim_y) * z
    zz = z_inv * z_inv
    jw0 = fx * z_inv[:, None] * R[0] - (fx * jx * zz)[:, None] * R[2]
    jw1 = fy * z_inv[:, None] * R[1] - (fy * jy * zz)[:, None] * R[2]
    M = quat_to_rotmat(quats) * scales[:, None, :]
    T0 = torch.einsum("nj,njk->nk", jw0, M)
    T1 = torch.einsum("nj,njk->nk", jw1, M)
    a = (T0 * T0).sum(1) + low_pass
    b = (T0 * T1).sum(1)
    c = (T1 * T1).sum(1) + low_pass
    det = a * c - b * b
    u = fx * p[:, 0] / z + cx
    v = fy * p[:, 1] / z + cy
    return torch.stack([u, v], 1), torch.stack([c / det, -b / det, a / det], 1)


def test_analytic_projection_backward_matches_autograd():
    s = scenes.config1(4, n=4000, channels=0)
    cam = s.cameras[0]
    # Add points beside and behind the camera so the clamp and near-plane branches are exercised.
    rng = np.random.default_rng(0)
    extra = rng.normal(0.0, 6.0, (1000, 3)).astype(np.float32)
    means = np.concatenate([s.means.numpy(), extra])
    scales = np.concatenate([s.scales.numpy(), np.exp(rng.normal(-3, 0.5, (1000, 3))).astype(np.float32)])
    quats = np.concatenate([s.quats.numpy(), s.quats.numpy()[:1000]])
    n = means.shape[0]
    w2c = cam.world_to_camera.numpy()
    args = (cam.fx, cam.fy, cam.cx, cam.cy, cam.width, cam.height)
    gm2 = rng.standard_normal((n, 2)).astype(np.float32)
    gcon = rng.standard_normal((n, 3)).astype(np.float32) * 1e-3
    got = oracle.project_backward(gm2, gcon, means, scales, quats, w2c, *args)

    tm = torch.tensor(means, dtype=torch.float64, requires_grad=True)
    ts = torch.tensor(scales, dtype=torch.float64, requires_grad=True)
    tq = torch.tensor(quats, dtype=torch.float64, requires_grad=True)
    m2, con = project_torch(tm, ts, tq, torch.tensor(w2c, dtype=torch.float64), *args)
    (m2 * torch.tensor(gm2, dtype=torch.float64)).sum().add_((con * torch.tensor(gcon, dtype=torch.float64)).sum()
                                                             ).backward()
    # Compare where the 2-D covariance is well conditioned (the reference falls back to a
    # non-inverse branch for det <= 0) and the point is not exactly on a clamp edge.
    p_cam = means @ w2c[:3, :3].T + w2c[:3, 3]
    ok = np.isfinite(con.detach().numpy()).all(1) & (np.abs(p_cam[:, 2] - 0.2) > 1e-3)
    assert ok.mean() > 0.9
    for name, g, w in (("means", got[0], tm.grad), ("scales", got[1], ts.grad), ("quats", got[2], tq.grad)):
        w = w.numpy()[ok]
        g = g[ok]
        scale = np.abs(w).max(axis=1, keepdims=True) + 1e-30
        err = np.abs(g - w) / scale
        assert np.quantile(err, 0.999) < 1e-3, f"{name}: 99.9% quantile relative error {np.quantile(err, 0.999):.2e}"
        assert np.median(err) < 1e-5, f"{name}: median relative error {np.median(err):.2e}"

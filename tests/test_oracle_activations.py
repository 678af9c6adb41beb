"""Pins the oracle's restatements of the torch glue around the path, on CPU, against the
reference's own composition of torch functions evaluated in float64:

* oracle.activate / activate_backward: the model's parameter activations of
  gaussian_splatting/utils/gaussian.py:73-98 (torch.exp of the log-scales, F.normalize of the
  quaternions, torch.sigmoid of the opacity logits) and their autograd gradients;
* oracle.view_dirs / view_dirs_backward: the viewing directions of utils/gaussian.py:110,
  F.normalize(means - camera_center, dim=-1), and their autograd gradient.

The oracle computes in float32 with one rounding per operation (its exp is oracle_expf), so the
forward values agree to a few float32 ulps and the gradients within the gradient tolerance.
"""
import numpy as np
import torch
import torch.nn.functional as F

import oracle
from helpers import assert_grads_close


def _params(n, seed):
    rng = np.random.default_rng(seed)
    log_scales = rng.normal(-3.5, 0.6, (n, 3)).astype(np.float32)
    quats = (rng.standard_normal((n, 4)) * rng.uniform(0.5, 2.0, (n, 1))).astype(np.float32)
    logits = rng.normal(0.0, 1.5, (n, 1)).astype(np.float32)
    return log_scales, quats, logits


def test_activate_matches_torch_float64():
    ls, q, lg = _params(4000, 0)
    scales, unit, opac = oracle.activate(ls, q, lg)
    t_ls, t_q, t_lg = (torch.from_numpy(a).double() for a in (ls, q, lg))
    np.testing.assert_allclose(scales, torch.exp(t_ls).numpy(), rtol=1e-6)
    np.testing.assert_allclose(unit, F.normalize(t_q, dim=-1).numpy(), rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(opac, torch.sigmoid(t_lg).numpy(), rtol=1e-6)


def test_activate_backward_matches_torch_autograd():
    ls, q, lg = _params(4000, 1)
    rng = np.random.default_rng(2)
    g_sc = rng.standard_normal(ls.shape).astype(np.float32)
    g_unit = rng.standard_normal(q.shape).astype(np.float32)
    g_op = rng.standard_normal(lg.shape).astype(np.float32)
    got = oracle.activate_backward(ls, q, lg, g_sc, g_unit, g_op)
    t = [torch.from_numpy(a).double().requires_grad_(True) for a in (ls, q, lg)]
    outs = (torch.exp(t[0]), F.normalize(t[1], dim=-1), torch.sigmoid(t[2]))
    torch.autograd.backward(outs, [torch.from_numpy(g).double() for g in (g_sc, g_unit, g_op)])
    for nm, a, b in zip(("log_scales", "quats", "logits"), got, t):
        assert_grads_close(a, b.grad.numpy(), nm, rel=1e-5)
    # Without an opacity gradient the logits get none.
    assert np.array_equal(oracle.activate_backward(ls, q, lg, g_sc, g_unit, None)[2], np.zeros_like(lg))


def test_activate_zero_quaternion_takes_the_clamp():
    """A zero quaternion normalises to zero (|q| clamped to 1e-12) and its gradient is g / 1e-12,
    as torch's F.normalize gives (the clamp's derivative is zero there)."""
    ls, q, lg = _params(3, 3)
    q[1] = 0.0
    _, unit, _ = oracle.activate(ls, q, lg)
    assert np.array_equal(unit[1], np.zeros(4, np.float32))
    g_unit = np.arange(12, dtype=np.float32).reshape(3, 4) + 1.0
    _, g_q, _ = oracle.activate_backward(ls, q, lg, np.zeros_like(ls), g_unit, None)
    assert np.array_equal(g_q[1], g_unit[1] / np.float32(1e-12))
    t = torch.from_numpy(q).double().requires_grad_(True)
    F.normalize(t, dim=-1).backward(torch.from_numpy(g_unit).double())
    np.testing.assert_allclose(g_q[1], t.grad[1].numpy(), rtol=1e-6)


def test_view_dirs_match_torch_normalize():
    rng = np.random.default_rng(4)
    center = rng.standard_normal(3).astype(np.float32)
    means = (center + 5.0 * rng.standard_normal((4000, 3))).astype(np.float32)
    dirs, s = oracle.view_dirs(means, center)
    t_m = torch.from_numpy(means).double().requires_grad_(True)
    ref = F.normalize(t_m - torch.from_numpy(center).double(), dim=-1)
    np.testing.assert_allclose(dirs, ref.detach().numpy(), rtol=1e-6, atol=1e-7)
    g = rng.standard_normal((4000, 3)).astype(np.float32)
    ref.backward(torch.from_numpy(g).double())
    assert_grads_close(oracle.view_dirs_backward(g, dirs, s), t_m.grad.numpy(), "means", rel=1e-5)

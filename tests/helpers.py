"""Shared comparison helpers for the parity tests (tolerances stated where they are used)."""
from __future__ import annotations

import math

import numpy as np

# Tolerances from the build's north star: RGB within 1e-5 absolute, feature images within 1e-3
# absolute (TF32), gradients within 1e-4 relative to the largest gradient of the tensor.
RGB_ATOL = 1e-5
FEATURE_ATOL = 1e-3
GRAD_REL = 1e-4


def seeded_uniform(seed: int, shape) -> np.ndarray:
    return np.random.default_rng(seed).random(shape, dtype=np.float32)


def assert_close_abs(got, want, atol: float, what: str = "", max_bad_fraction: float = 0.0) -> None:
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    if want.size == 0:
        return
    diff = np.abs(got - want)
    bad = diff > atol
    frac = bad.mean()
    assert frac <= max_bad_fraction, (
        f"{what}: {bad.sum()} of {bad.size} beyond {atol:g} (max {diff.max():.3e} at "
        f"{np.unravel_index(diff.argmax(), diff.shape)})")


def assert_grads_close(got, want, what: str = "", rel: float = GRAD_REL, max_bad_fraction: float = 1e-3,
                       max_rel: float = 2e-3) -> None:
    """|got - want| <= rel * max|want| + 1e-3 * |want| for all but max_bad_fraction of entries
    (a pair sitting exactly on the MIN_ALPHA / MIN_T cutoff may flip between precisions), and
    no entry worse than max_rel * max|want|."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    if want.size == 0:
        return
    scale = np.abs(want).max()
    if scale == 0:
        assert np.abs(got).max() == 0, f"{what}: expected all zeros"
        return
    diff = np.abs(got - want)
    bad = diff > rel * scale + 1e-3 * np.abs(want)
    assert bad.mean() <= max_bad_fraction, (
        f"{what}: {bad.sum()} of {bad.size} outside {rel:g} of max {scale:.3e} (worst {diff.max() / scale:.3e})")
    assert diff.max() <= max_rel * scale, f"{what}: worst error {diff.max() / scale:.3e} of max"


def perc(x, q):
    x = np.sort(np.abs(np.asarray(x)).ravel())
    return x[max(0, math.ceil(q * x.size) - 1)] if x.size else 0.0

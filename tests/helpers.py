"""Shared comparison helpers for the parity tests (tolerances stated where they are used).

Every gradient comparison records its worst error relative to the largest reference entry; the
session prints them all at the end (tests/conftest.py), so the achieved precision is visible
whether or not a bound is close."""
from __future__ import annotations

import math

import numpy as np

# Tolerances from the build's north star: RGB within 1e-5 absolute, feature images within 1e-3
# absolute, gradients within 1e-4 relative (every entry within 1e-4 of the tensor's largest
# reference entry).
RGB_ATOL = 1e-5
FEATURE_ATOL = 1e-3
GRAD_REL = 1e-4

# (label, worst |got - want| / max |want|, entries) of every gradient compared this session, and
# (label, worst |got - want|) of every absolute comparison.
GRAD_REPORT: list[tuple[str, float, int]] = []
ABS_REPORT: list[tuple[str, float, float]] = []
_current_test = {"id": ""}


def set_current_test(node_id: str) -> None:
    _current_test["id"] = node_id


def seeded_uniform(seed: int, shape) -> np.ndarray:
    return np.random.default_rng(seed).random(shape, dtype=np.float32)


def assert_close_abs(got, want, atol: float, what: str = "") -> None:
    """Every entry within atol of the reference (no exceptions)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    if want.size == 0:
        return
    diff = np.abs(got - want)
    worst = float(diff.max())
    ABS_REPORT.append((f"{_current_test['id']} {what}", worst, atol))
    bad = diff > atol
    assert not bad.any(), (
        f"{what}: {bad.sum()} of {bad.size} beyond {atol:g} (max {worst:.3e} at "
        f"{np.unravel_index(diff.argmax(), diff.shape)})")


def grad_rel_error(got, want) -> float:
    """max |got - want| / max |want| (0 for two all-zero tensors)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    scale = np.abs(want).max() if want.size else 0.0
    if scale == 0:
        return 0.0 if (got.size == 0 or np.abs(got).max() == 0) else math.inf
    return float(np.abs(got - want).max() / scale)


def assert_grads_close(got, want, what: str = "", rel: float = GRAD_REL) -> None:
    """|got - want| <= rel * max|want| for every entry: the north star's 1e-4 relative bound on FP32
    gradients, relative to the tensor's largest entry (entries sum float atomics in any order, so
    single small entries carry the rounding of large ones).  Records the worst relative error."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    if want.size == 0:
        return
    worst = grad_rel_error(got, want)
    GRAD_REPORT.append((f"{_current_test['id']} {what}", worst, int(want.size)))
    if np.abs(want).max() == 0:
        assert worst == 0.0, f"{what}: expected all zeros"
        return
    scale = np.abs(want).max()
    diff = np.abs(got - want)
    bad = diff > rel * scale
    assert not bad.any(), (
        f"{what}: {bad.sum()} of {bad.size} entries outside {rel:g} of max {scale:.3e} (worst {worst:.3e} at "
        f"{np.unravel_index(diff.argmax(), diff.shape)})")


def assert_close_fastmath(got, want, atol: float, what: str = "", max_bad_fraction: float = 1e-3) -> None:
    """For comparisons with the reference's own CUDA build only: it compiles with --use_fast_math, so its
    alpha uses an approximate exponential and a pair within rounding of the MIN_ALPHA cutoff can land on
    the other side of it.  At most max_bad_fraction of the entries may then exceed atol."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    if want.size == 0:
        return
    diff = np.abs(got - want)
    bad = diff > atol
    ABS_REPORT.append((f"{_current_test['id']} {what} (vs fast-math build, {bad.mean():.1e} beyond)",
                       float(diff.max()), atol))
    assert bad.mean() <= max_bad_fraction, f"{what}: {bad.sum()} of {bad.size} beyond {atol:g}"


def assert_grads_close_fastmath(got, want, what: str = "", rel: float = GRAD_REL, max_bad_fraction: float = 1e-3,
                                max_rel: float = 2e-3) -> None:
    """Gradients against the reference's own fast-math CUDA build (see assert_close_fastmath): within
    rel of the largest entry for all but max_bad_fraction of the entries (the gaussians of a pair that
    flipped at the MIN_ALPHA cutoff), and none beyond max_rel of it."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    if want.size == 0:
        return
    worst = grad_rel_error(got, want)
    GRAD_REPORT.append((f"{_current_test['id']} {what} (vs fast-math build)", worst, int(want.size)))
    scale = np.abs(want).max()
    if scale == 0:
        assert worst == 0.0, f"{what}: expected all zeros"
        return
    bad = np.abs(got - want) > rel * scale
    assert bad.mean() <= max_bad_fraction, f"{what}: {bad.sum()} of {bad.size} outside {rel:g} of max"
    assert worst <= max_rel, f"{what}: worst error {worst:.3e} of max"


def perc(x, q):
    x = np.sort(np.abs(np.asarray(x)).ravel())
    return x[max(0, math.ceil(q * x.size) - 1)] if x.size else 0.0

"""Shared helpers of the test suite (inputs, error metric, library handles)."""
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")

# Parity bar of the hot path: per-element relative error <= 1e-3 against the
# reference's float32 CPU vec_dot.  The denominator is floored at 1e-2 of the
# output's RMS: outputs that cancel to ~0 carry the float32 summation noise of
# the reference itself (~1e-6 * rms for 11008-term rows), which a pure
# per-element relative bar would charge to the GPU.  Tests pair this with a
# check that the GPU is at least as close to the float64-exact product as
# the reference is.
REL_TOL = 1e-3
RMS_FLOOR = 1e-2


def rel_err(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    rms = np.sqrt(np.mean(ref * ref)) if ref.size else 0.0
    den = np.maximum(np.abs(ref), RMS_FLOOR * rms)
    den = np.where(den == 0, 1.0, den)
    return np.abs(y - ref) / den


def plain_rel_err(y, ref):
    """Per-element |y - ref| / |ref| with no floor (0 where both are 0)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    d = np.abs(y - ref)
    with np.errstate(divide="ignore", invalid="ignore"):
        e = np.where(d == 0, 0.0, d / np.abs(ref))
    return e


def parity_line(y, ref, absdot=None, what=""):
    """One line reporting both figures: the floored per-element relative
    error (the bar) and the plain per-element relative error, with, given
    absdot = sum_k |w[r,k] x[k]| per row, the condition number
    absdot / |ref| of the row where the plain error is largest -- how much
    cancellation amplifies the float32 rounding there."""
    fl = rel_err(y, ref)
    pl = plain_rel_err(y, ref)
    if not pl.size:
        return f"{what}: empty"
    i = int(np.argmax(pl))
    line = f"{what}: max rel err {fl.max():.2e} (floored), plain {pl[i]:.2e} at row {i}"
    if absdot is not None:
        r = abs(float(np.asarray(ref, np.float64)[i]))
        kappa = float(absdot[i]) / r if r > 0 else float("inf")
        line += f" (condition number {kappa:.3g})"
    return line


def assert_parity(y, ref, tol=REL_TOL, what="", absdot=None):
    e = rel_err(y, ref)
    worst = int(np.argmax(e)) if e.size else 0
    assert e.size == 0 or e.max() <= tol, (
        f"{what}: max rel err {e.max():.3e} at {worst} (y={y[worst]!r}, ref={ref[worst]!r})")
    print(parity_line(y, ref, absdot, what))
    return float(e.max()) if e.size else 0.0


def seeded_weights(seed, rows, cols, std=0.02):
    return np.random.default_rng(seed).normal(0.0, std, size=(rows, cols)).astype(np.float32)


def seeded_x(seed, n):
    return np.random.default_rng(seed).normal(0.0, 1.0, size=n).astype(np.float32)

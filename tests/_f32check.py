"""Shared checks for the fp32 paths (imported by the fp32 GPU tests)."""
import numpy as np


def all_within(got, want, tol, floor=0.0):
    """The reference gate (mlx/scripts/harness.py:26-33): every element
    within tol + tol*|want| (+ an absolute noise floor)."""
    err = np.abs(got.astype(np.float64) - want)
    bad = err > tol + floor + tol * np.abs(want)
    assert not bad.any(), (int(bad.sum()), float(err.max()))


def check_against_fp32_golden(got, golden, exact, tol):
    """The golden is the reference hook run in fp32; with N(0,1) weights its
    outputs reach ~1e4 (rms ~1400) and its own rounding error is up to ~0.4,
    i.e. 2.6e-4 of the rms, against float64: an output formed by cancelling
    terms of that size carries fp32 noise of that order whatever its own
    magnitude. So: every element within tol (+ a floor of 1e-4 of the rms)
    of the float64 oracle, and within tol of the golden up to the golden's
    own largest error."""
    rms = float(np.sqrt(np.mean(np.square(exact, dtype=np.float64))))
    all_within(got, exact, tol, floor=1e-4 * rms)
    own = float(np.abs(golden.astype(np.float64) - exact).max())
    err = np.abs(got.astype(np.float64) - golden)
    assert np.all(err <= tol + own + tol * np.abs(golden)), (float(err.max()), own)



"""Tolerances shared by the CPU and GPU parity tests.

The bar for floating-point outputs is max-abs 2e-2 and mean relative 5e-3,
with fp32 accumulation; the relative error is averaged over elements whose
reference magnitude is at least 1e-2 (smaller ones are covered by max-abs)."""
import numpy as np

MAX_ABS = 2e-2
MEAN_REL = 5e-3


def errors(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    diff = np.abs(got - ref)
    big = np.abs(ref) >= 1e-2
    rel = float((diff[big] / np.abs(ref[big])).mean()) if big.any() else 0.0
    return float(diff.max()) if diff.size else 0.0, rel


def assert_close(got, ref, act=None, max_abs=MAX_ABS, mean_rel=MEAN_REL):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.array_equal(np.isnan(got), np.isnan(ref)), "NaN pattern differs"
    m = ~np.isnan(ref)
    mx, rel = errors(got[m], ref[m])
    assert mx <= max_abs and rel <= mean_rel, f"max_abs={mx:.3e} mean_rel={rel:.3e}"
    return mx, rel

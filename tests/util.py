"""Shared test helpers (tolerances are written here, once)."""
import numpy as np

# north_star: per-op fp32 outputs within 1e-3 relative error.  Elementwise:
# |a - b| <= RTOL * |b| + RTOL * 1e-2 * max|b|  (the second term only matters
# for entries that cancel to ~0, where a relative bound is meaningless).
RTOL = 1e-3


def assert_rel(actual, desired, rtol=RTOL, what=""):
    a = np.asarray(actual, np.float64)
    b = np.asarray(desired, np.float64)
    assert a.shape == b.shape, (a.shape, b.shape)
    assert np.all(np.isfinite(a)), f"{what}: non-finite output"
    scale = np.max(np.abs(b)) if b.size else 0.0
    err = np.abs(a - b)
    bound = rtol * np.abs(b) + rtol * 1e-2 * scale
    bad = err > bound
    if bad.any():
        i = int(np.argmax(err - bound))
        raise AssertionError(f"{what}: {bad.sum()} / {b.size} outside rtol={rtol}; worst idx {i}: "
                             f"{a.flat[i]} vs {b.flat[i]} (max|b|={scale})")


def max_rel_err(actual, desired):
    a = np.asarray(actual, np.float64)
    b = np.asarray(desired, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))

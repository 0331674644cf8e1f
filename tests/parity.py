"""Shared parity helpers for the GPU tests.

Tolerance (north star): floating outputs agree with the CPU oracle within a
max relative error of 1e-2 with fp32 accumulation, where
    rel_i = |a_i - r_i| / max(|r_i|, rms(r))
(the rms floor keeps near-zero entries from dominating; the reference's own
convention |a - e| <= max(|e|, 1) * tol, weights/parity_tests.rs:1734, is the
same idea with a floor of 1). Integer outputs (nibbles, route ids) are
bit-exact.
"""

import numpy as np

REL_TOL = 1e-2


def max_rel(actual, ref) -> float:
    a = np.asarray(actual, np.float64).ravel()
    r = np.asarray(ref, np.float64).ravel()
    assert a.shape == r.shape
    if r.size == 0:
        return 0.0
    rms = float(np.sqrt(np.mean(r * r)))
    denom = np.maximum(np.abs(r), rms if rms > 0 else 1.0)
    return float(np.max(np.abs(a - r) / denom))


def assert_close(actual, ref, tol=REL_TOL, what=""):
    m = max_rel(actual, ref)
    assert np.all(np.isfinite(np.asarray(actual, np.float64))), f"{what}: non-finite output"
    assert m <= tol, f"{what}: max relative error {m:.3e} > {tol:.1e}"
    return m

"""Correctly rounded float32 ``exp2`` for the CPU oracle (test infrastructure).

The reference computes ``exp(x)`` as ``np.exp2(f32(x * log2e))`` in float32
(``tools/ref_qwen3.py:27-29``).  numpy's float32 ``exp2`` is dispatched by CPU
feature: on an AVX-512 host it differs from the correctly rounded result by one
ulp on about a fifth of all inputs, and without AVX-512 it follows glibc.  The
reference's value is therefore host dependent.  The parity target used by this
build is the host-independent one, the correctly rounded ``RN_f32(2^x)``; the
device kernels implement the same function.

Method: ``y = exp2_f64(x)`` (numpy float64, error far below 2^-46 relative),
``RN_f32(y)`` is the answer unless ``y`` is within ``2^-44 * y`` of a midpoint
between two adjacent float32 values; those rare inputs are resolved exactly
with mpmath at 200 bits (ties, which only occur at x = -150, go to even).
"""

from __future__ import annotations

import numpy as np

_THRESH = 2.0 ** -44


def _resolve_one(x: float) -> np.float32:
    import mpmath
    mpmath.mp.prec = 200
    t = mpmath.power(2, mpmath.mpf(float(x)))
    with np.errstate(over="ignore", under="ignore"):
        r = np.float32(np.exp2(np.float64(x)))
    cands = {float(r), float(np.nextafter(r, np.float32(np.inf))),
             float(np.nextafter(r, np.float32(-np.inf)))}
    best = None
    for c in cands:
        if not np.isfinite(c):
            continue
        d = abs(mpmath.mpf(c) - t)
        bits = int(np.float32(c).view(np.uint32))
        key = (d, bits & 1)
        if best is None or key < best[0]:
            best = (key, np.float32(c))
    return best[1]


def exp2_cr(x) -> np.ndarray:
    """Correctly rounded float32 2^x for a float32 array (any shape)."""
    x = np.asarray(x, dtype=np.float32)
    x64 = x.astype(np.float64)
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        y = np.exp2(x64)
        r = y.astype(np.float32)
        r64 = r.astype(np.float64)
        up = np.nextafter(r, np.float32(np.inf)).astype(np.float64)
        dn = np.nextafter(r, np.float32(-np.inf)).astype(np.float64)
        mid = np.where(y >= r64, (r64 + up) * 0.5, (r64 + dn) * 0.5)
        hard = np.isfinite(y) & (y > 0) & np.isfinite(mid) & (np.abs(y - mid) <= y * _THRESH)
    if np.any(hard):
        r = r.copy()
        idx = np.nonzero(hard)
        for pos in zip(*idx):
            r[pos] = _resolve_one(float(x[pos]))
    return r


def exp2_numpy_f32(x) -> np.ndarray:
    """The reference's own float32 ``np.exp2`` (host-dependent rounding)."""
    return np.exp2(np.asarray(x, dtype=np.float32)).astype(np.float32)

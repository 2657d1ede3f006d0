"""Host-side checks of arithmetic identities the CUDA kernels rely on,
restated in numpy (no GPU needed)."""

from __future__ import annotations

import numpy as np


def _fma32(a, b, c):
    """Correctly rounded float32 fma(a, b, c): a*b is exact in float64, the
    addition's float64 rounding error is recovered by two-sum, and the final
    rounding to float32 picks the nearest of the three float32 candidates
    around the float64 sum."""
    p = a.astype(np.float64) * b.astype(np.float64)
    c64 = c.astype(np.float64)
    s = p + c64
    bb = s - p
    err = (p - (s - bb)) + (c64 - bb)
    r = s.astype(np.float32)
    up = np.nextafter(r, np.float32(np.inf))
    dn = np.nextafter(r, np.float32(-np.inf))
    d_r = np.abs((r.astype(np.float64) - s) - err)
    d_up = np.abs((up.astype(np.float64) - s) - err)
    d_dn = np.abs((dn.astype(np.float64) - s) - err)
    out = np.where(d_up < d_r, up, r)
    return np.where(d_dn < np.minimum(d_r, d_up), dn, out)


def test_corrected_reciprocal_division_is_ieee_division():
    """The prefill epilogue quantises x / scale as q0 = x * rs, r = fma(-q0,
    scale, x), q = r == 0 ? q0 : fma(r, rs, q0) with rs = RN(1/scale)
    (Markstein's correction). Over the quantiser's domain (scale = max(amax,1e-10)/448,
    |x| <= amax) that must equal IEEE float32 division bit for bit."""
    rng = np.random.default_rng(0)
    n = 400_000
    f32 = np.float32
    amax = (rng.uniform(0.5, 1.0, n) * 2.0 ** rng.integers(-40, 30, n)).astype(f32)
    x = (amax * rng.uniform(-1, 1, n)).astype(f32)
    x[:500], x[500:1000] = amax[:500], -amax[500:1000]      # the group maximum itself
    x[1000:1500] = (amax[1000:1500] * f32(2.0 ** -20)).astype(f32)  # tiny members
    x[1500:1600], x[1600:1700] = f32(0.0), f32(-0.0)  # signed zeros keep their sign
    sc = (np.maximum(amax, f32(1e-10)) / f32(448)).astype(f32)
    rs = (f32(1) / sc).astype(f32)
    ieee = (x / sc).astype(f32)
    q0 = (x * rs).astype(f32)
    r = _fma32(-q0, sc, x)
    q = np.where(r == 0, q0, _fma32(r, rs, q0))
    np.testing.assert_array_equal(q.view(np.uint32), ieee.view(np.uint32))
    assert (q0 != ieee).any()  # the correction is doing work

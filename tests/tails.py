"""Saturated-tail truth for the stable tanh jet, from 100-digit mpmath (the method of the
reference's tests/test_jet_stable.py:28-42).

For a jet whose input has order-0 value ``center`` and first-order coefficient 1 along
every axis (``z = center + x + y (+ t)``), the Taylor coefficient of ``tanh(z)`` at
multi-index alpha is ``tanh^(|alpha|)(center) / prod(alpha_i!)``.
"""

import math
from functools import lru_cache

import numpy as np

CENTERS = (0.0, 5.0, 20.0, -20.0, 100.0, 350.0)


@lru_cache(maxsize=None)
def tanh_derivative(center, order):
    import mpmath as mp
    with mp.workdps(100):
        return float(mp.diff(mp.tanh, mp.mpf(center), order, addprec=1200))


def input_jets(dim, centers=CENTERS):
    """``[len(centers), Q, 1]`` input jets with unit first-order coefficients on every axis."""
    from oracle import jets as J
    z = np.zeros((len(centers), J.q(dim), 1))
    z[:, 0, 0] = centers
    for axis in range(dim):
        z[:, J.unit(dim, axis), 0] = 1.0
    return z


def expected_jets(dim, centers=CENTERS):
    from oracle import jets as J
    out = np.zeros((len(centers), J.q(dim), 1))
    for i, c in enumerate(centers):
        for k, alpha in enumerate(J.basis(dim)):
            out[i, k, 0] = tanh_derivative(c, sum(alpha)) / math.prod(math.factorial(a) for a in alpha)
    return out


FOURTH_CENTERS = (0.0, 0.3, -0.7, 15.0, 20.0)
A1_PROBES = (0.0, 15.0, 20.0, 21.0, 40.0, 100.0, 300.0, 355.0, 360.0, 370.0, 372.0, 373.0, 374.0, 380.0)


def fourth_derivative_case(centers=FOURTH_CENTERS):
    """2-D input jets ``z = z0 + x`` and a seed on the x^3 coefficient: the VJP's order-0
    entry is d/dz0 of tanh'''(z0)/6 = tanh''''(z0)/6 (the reference's
    sources/flashns_v8_reference/tests/verify_math.py:127-139).  Returns (z, seed, expected)."""
    import mpmath as mp
    from oracle import jets as J
    z = np.zeros((len(centers), J.q(2), 1))
    z[:, 0, 0] = centers
    z[:, J.unit(2, 0), 0] = 1.0
    seed = np.zeros_like(z)
    seed[:, J.index(2)[(3, 0)], 0] = 1.0
    expected = []
    with mp.workdps(100):
        for c in centers:
            t = mp.tanh(mp.mpf(c))
            expected.append(float((16 * t - 24 * t ** 3) * (1 - t * t) / 6))
    return z, seed, np.array(expected)


def a1_truth(z):
    """sech^2 z as (2r / (1 + r^2))^2, r = exp(-|z|), at 420 digits (verify_math.py:186-197)."""
    import mpmath as mp
    with mp.workdps(420):
        r = mp.exp(-abs(mp.mpf(z)))
        return (2 * r / (1 + r * r)) ** 2


def a1_tail_ok(actual, z, quanta=2):
    """Relative error < 5e-13 where sech^2 z is a normal double; otherwise at most
    ``quanta`` subnormal quanta of absolute error (the reference's scalar criterion)."""
    import mpmath as mp
    expected = a1_truth(z)
    with mp.workdps(420):
        err = abs(mp.mpf(float(actual)) - expected)
        if expected >= mp.mpf(np.finfo(np.float64).tiny):
            return float(err / expected) < 5e-13
        return err <= quanta * mp.mpf(float(np.nextafter(0.0, 1.0)))


def within_tail_tolerance(actual, expected):
    """|a - e| <= 1e-11 |e| + 8 ulp(e), elementwise (the reference's tail criterion)."""
    actual, expected = np.asarray(actual, dtype=np.float64), np.asarray(expected, dtype=np.float64)
    ulp = np.vectorize(math.ulp)(expected)
    return np.abs(actual - expected) <= 1e-11 * np.abs(expected) + 8 * ulp

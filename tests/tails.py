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


def within_tail_tolerance(actual, expected):
    """|a - e| <= 1e-11 |e| + 8 ulp(e), elementwise (the reference's tail criterion)."""
    actual, expected = np.asarray(actual, dtype=np.float64), np.asarray(expected, dtype=np.float64)
    ulp = np.vectorize(math.ulp)(expected)
    return np.abs(actual - expected) <= 1e-11 * np.abs(expected) + 8 * ulp

"""Factorial-normalized Taylor jets, truncated Cauchy products, stable tanh jets.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

A jet row-block stores ``c_alpha = d^alpha f / alpha!`` for every multi-index
``alpha`` with ``|alpha| <= order``, in the canonical order of
``src/flashns/jet_spec.py:30-41`` (sorted by ``(|alpha|, alpha)``).  Because the
order is sorted by total degree first, the order-k basis is a prefix of the
order-3 basis; truncating a jet to order k keeps its first ``q(dim, k)`` rows.
"""

from functools import lru_cache
from itertools import product
from math import factorial, prod

import numpy as np


@lru_cache(None)
def basis(dim, order=3):
    """Canonical multi-indices (``src/flashns/jet_spec.py:30-41``), truncated."""
    full = sorted((a for a in product(range(4), repeat=dim) if sum(a) <= 3),
                  key=lambda a: (sum(a), a))
    return tuple(a for a in full if sum(a) <= order)


def q(dim, order=3):
    return len(basis(dim, order))


@lru_cache(None)
def index(dim):
    return {a: i for i, a in enumerate(basis(dim, 3))}


@lru_cache(None)
def recovery(dim, order=3):
    """``prod(alpha!)`` per coefficient (``src/flashns/jet_spec.py:48-49``)."""
    return np.array([prod(factorial(v) for v in a) for a in basis(dim, order)], dtype=np.float64)


def unit(dim, axis):
    """Row of the first-order coefficient along ``axis`` (reverse axis order)."""
    return index(dim)[tuple(int(axis == j) for j in range(dim))]


@lru_cache(None)
def pairs(dim, order=3):
    """For each gamma: the (i, j) with alpha_i + alpha_j = gamma.

    Same relation as ``product_pairs`` (``src/flashns/jet_stable.py:37-49``).
    """
    b = basis(dim, order)
    lookup = {a: i for i, a in enumerate(b)}
    out = []
    for g in b:
        terms = []
        for i, a in enumerate(b):
            if all(x <= y for x, y in zip(a, g)):
                terms.append((i, lookup[tuple(y - x for x, y in zip(a, g))]))
        out.append(tuple(terms))
    return tuple(out)


def cauchy(a, b, dim, order):
    """Truncated product of jets stored on axis 1: ``[N, q, C]``."""
    out = np.zeros_like(a)
    for g, terms in enumerate(pairs(dim, order)):
        acc = np.zeros_like(a[:, 0])
        for i, j in terms:
            acc = acc + a[:, i] * b[:, j]
        out[:, g] = acc
    return out


def stable_a1(z0):
    """``sech^2`` from ``r = exp(-|z|)`` (``src/flashns/jet_packed.py:62-64``)."""
    r = np.exp(-np.abs(z0))
    v = (2.0 * r) / (1.0 + r * r)
    return v * v


def tanh_jet(z, dim, order=3):
    """Stable tanh composition of a jet ``z[N, q, C]`` (``jet_stable.py:62-76``).

    ``h = a1*delta - t*a1*delta^2 + a1*(t^2 - 1/3)*delta^3`` with ``h_0 = tanh z_0``
    and the stored auxiliary ``a1 = sech^2 z_0``.
    """
    z0 = z[:, 0]
    t = np.tanh(z0)
    a1 = stable_a1(z0)
    if z.shape[1] == 1:
        return t[:, None].copy(), a1
    delta = z.copy()
    delta[:, 0] = 0.0
    p2 = cauchy(delta, delta, dim, order)
    p3 = cauchy(p2, delta, dim, order)
    h = a1[:, None] * delta - (t * a1)[:, None] * p2 + (a1 * (t * t - 1.0 / 3.0))[:, None] * p3
    h[:, 0] = t
    return h, a1


def tanh_vjp(h, a1, hbar, dim, order=3):
    """Transpose of the jet Jacobian (``src/flashns/jet_packed.py:76-88``).

    ``g = -(H*H)`` except ``g_0 = a1``; ``zbar_beta = sum_{alpha>=beta} hbar_alpha g_{alpha-beta}``.
    """
    if h.shape[1] == 1:
        return hbar * a1[:, None]
    g = -cauchy(h, h, dim, order)
    g[:, 0] = a1
    out = np.zeros_like(h)
    for alpha, terms in enumerate(pairs(dim, order)):
        for beta, gamma in terms:
            out[:, beta] += hbar[:, alpha] * g[:, gamma]
    return out

"""Navier-Stokes residual polynomials and their explicit seeds (CPU, NumPy).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Each residual is a polynomial in raw derivatives ``D(field, alpha)`` written
from the PDE; the differentiated residuals of the gradient-enhanced (u, v, p)
objective are produced by applying the Leibniz rule to those polynomials.
Raw derivatives are ``alpha! * c_alpha`` (``src/flashns/jet_spec.py:48-57``).

Heads
-----
``uvp``  -- the reference objective, ``src/flashns/ns_seed.py:26-87``: fields
          (u, v, p), residuals (ru, rv, div, dx ru, dx rv, dx div, dy ru, dy rv,
          dy div), loss ``0.5*w*(sum r_0..2^2 + gamma*sum r_3..8^2)``.
``psi``  -- stream-function head (not in the reference): outputs (psi, p),
          u = psi_y, v = -psi_x, so continuity holds identically; residuals
          (ru, rv); in 3-D the third axis is time and ``u_t``, ``v_t`` are added.
          Loss ``0.5*w*(ru^2 + rv^2)``.
"""

from functools import lru_cache
from math import factorial, prod

import numpy as np

from oracle.jets import index, q

# An expression is a dict {factors: coefficient}; factors is a sorted tuple of
# (field, alpha) pairs (at most two for these PDEs); the empty tuple is a constant.


def _e(dim, *axes):
    a = [0] * dim
    for x in axes:
        a[x] += 1
    return tuple(a)


def lin(terms):
    """Linear expression from [(coefficient, field, alpha)]."""
    out = {}
    for c, f, a in terms:
        key = ((f, a),)
        out[key] = out.get(key, 0.0) + c
    return out


def add(*exprs):
    out = {}
    for e in exprs:
        for k, c in e.items():
            out[k] = out.get(k, 0.0) + c
    return {k: c for k, c in out.items() if c != 0.0}


def scale(e, s):
    return {k: c * s for k, c in e.items()}


def mul(x, y):
    out = {}
    for kx, cx in x.items():
        for ky, cy in y.items():
            k = tuple(sorted(kx + ky))
            out[k] = out.get(k, 0.0) + cx * cy
    return {k: c for k, c in out.items() if c != 0.0}


def diff(e, axis):
    """Leibniz rule: d/dx_axis of a polynomial in raw derivatives."""
    out = {}
    for k, c in e.items():
        for pos, (f, a) in enumerate(k):
            b = list(a)
            b[axis] += 1
            nk = tuple(sorted(k[:pos] + ((f, tuple(b)),) + k[pos + 1:]))
            out[nk] = out.get(nk, 0.0) + c
    return {k: c for k, c in out.items() if c != 0.0}


def d_of(e, axis):
    return diff(e, axis)


def uvp_residuals(nu, gamma):
    """Residual polynomials + scales of the reference (u, v, p) objective.

    Order and weights follow ``src/flashns/ns_seed.py:26-43,67-69``.
    """
    dim, X, Y = 2, 0, 1
    U = lambda *ax: lin([(1.0, 0, _e(dim, *ax))])
    V = lambda *ax: lin([(1.0, 1, _e(dim, *ax))])
    P = lambda *ax: lin([(1.0, 2, _e(dim, *ax))])
    ru = add(mul(U(), U(X)), mul(V(), U(Y)), P(X), scale(add(U(X, X), U(Y, Y)), -nu))
    rv = add(mul(U(), V(X)), mul(V(), V(Y)), P(Y), scale(add(V(X, X), V(Y, Y)), -nu))
    div = add(U(X), V(Y))
    base = [ru, rv, div]
    res = base + [diff(r, X) for r in base] + [diff(r, Y) for r in base]
    return res, [1.0] * 3 + [gamma] * 6


def psi_residuals(nu, dim):
    """Momentum residuals of the stream-function head.

    u = psi_y, v = -psi_x.  ``ru = u u_x + v u_y + p_x - nu (u_xx + u_yy) [+ u_t]``,
    ``rv = u v_x + v v_y + p_y - nu (v_xx + v_yy) [+ v_t]``; axis 2 is time.
    """
    X, Y = 0, 1
    S = lambda c, *ax: lin([(c, 0, _e(dim, *ax))])
    P = lambda *ax: lin([(1.0, 1, _e(dim, *ax))])
    u = lambda *ax: S(1.0, Y, *ax)
    v = lambda *ax: S(-1.0, X, *ax)
    ru = add(mul(u(), u(X)), mul(v(), u(Y)), P(X), scale(add(u(X, X), u(Y, Y)), -nu))
    rv = add(mul(u(), v(X)), mul(v(), v(Y)), P(Y), scale(add(v(X, X), v(Y, Y)), -nu))
    if dim == 3:
        ru = add(ru, u(2))
        rv = add(rv, v(2))
    return [ru, rv], [1.0, 1.0]


@lru_cache(None)
def residual_program(head, dim, nu, gamma):
    """Residuals in coefficient space: list of [(coef, ((field, row), ...))]."""
    if head == "uvp":
        if dim != 2:
            raise ValueError("the (u, v, p) head is 2-D only")
        res, scales = uvp_residuals(nu, gamma)
    elif head == "psi":
        res, scales = psi_residuals(nu, dim)
    else:
        raise ValueError("unknown head")
    idx = index(dim)
    program = []
    for r in res:
        terms = []
        for k, c in sorted(r.items()):
            factor = c
            rows = []
            for f, a in k:
                if sum(a) > 3:
                    raise ValueError("residual needs derivatives beyond third order")
                factor *= prod(factorial(v) for v in a)
                rows.append((f, idx[a]))
            terms.append((factor, tuple(rows)))
        program.append(terms)
    return tuple(program), tuple(scales)


def interior_seed(jets, weights, head, nu, gamma=0.2):
    """Loss and seed of the interior objective for jets ``[N, Q, F]``.

    Explicit first-order transpose in the manner of ``src/flashns/ns_seed.py:72-87``.
    Returns ``(loss_per_point[N], seed[N, Q, F])``.
    """
    n, qq, nf = jets.shape
    dim = 2 if qq == 10 else 3
    program, scales = residual_program(head, dim, float(nu), float(gamma))
    seed = np.zeros_like(jets)
    loss = np.zeros(n)
    for terms, s in zip(program, scales):
        r = np.zeros(n)
        for c, rows in terms:
            val = np.full(n, c)
            for f, i in rows:
                val = val * jets[:, i, f]
            r = r + val
        dr = weights * s * r
        loss = loss + 0.5 * dr * r
        for c, rows in terms:
            for pos, (f, i) in enumerate(rows):
                val = c * dr
                for other, (g, j) in enumerate(rows):
                    if other != pos:
                        val = val * jets[:, j, g]
                seed[:, i, f] += val
    return loss, seed


def residual_values(jets, head, nu, gamma=0.2):
    n, qq, _ = jets.shape
    dim = 2 if qq == 10 else 3
    program, _ = residual_program(head, dim, float(nu), float(gamma))
    out = np.zeros((n, len(program)))
    for k, terms in enumerate(program):
        for c, rows in terms:
            val = np.full(n, c)
            for f, i in rows:
                val = val * jets[:, i, f]
            out[:, k] += val
    return out


def boundary_fields(rows, head, dim, order):
    """Boundary fields from boundary rows ``[Nb, qb, Cout]``.

    Order 0: the raw network outputs.  Order 1 with the psi head: (u, v, p) =
    (psi_y, -psi_x, p) from the first-order coefficients.
    """
    if order == 0:
        return rows[:, 0, :]
    if head != "psi":
        raise ValueError("first-order boundary rows are defined for the psi head")
    uy, ux = index(dim)[tuple(int(j == 1) for j in range(dim))], index(dim)[tuple(int(j == 0) for j in range(dim))]
    return np.stack((rows[:, uy, 0], -rows[:, ux, 0], rows[:, 0, 1]), axis=1)


def boundary_seed(rows, weights, target, bc, head, dim, order):
    """Loss ``bc * sum w (f - f*)^2`` and its seed on the boundary rows."""
    fields = boundary_fields(rows, head, dim, order)
    err = fields - target
    loss = bc * (weights * err * err).sum(1)
    g = 2.0 * bc * weights * err
    seed = np.zeros_like(rows)
    if order == 0:
        seed[:, 0, :] = g
    else:
        uy = index(dim)[tuple(int(j == 1) for j in range(dim))]
        ux = index(dim)[tuple(int(j == 0) for j in range(dim))]
        seed[:, uy, 0] = g[:, 0]
        seed[:, ux, 0] = -g[:, 1]
        seed[:, 0, 1] = g[:, 2]
    return loss, seed

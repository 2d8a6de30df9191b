"""Packed loss + parameter-gradient evaluation on the CPU (NumPy FP64).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates ``PackedPINN.__call__`` (``src/flashns/pinn_packed.py:93-191``) for the
compact layout: one row space ``[interior points * Q ; boundary points * qb]``,
one GEMM per affine role, bias only on order-0 rows (``:120-121``), the stable
tanh jet per segment (``src/flashns/jet_packed.py:103-117``), the residual seed
(``src/flashns/ns_seed.py:72-87``, ``pinn_packed.py:150-153``) and the manual
reverse pass (``pinn_packed.py:155-190``).  Generalised to 2-D/3-D jets, the
stream-function head and first-order boundary rows (``boundary_order=1``).
"""

from concurrent.futures import ThreadPoolExecutor

import numpy as np

from oracle import jets as J
from oracle import residuals as RS


def coordinate_jets(x, ni, boundary_order):
    """Input jets of the coordinates (``src/flashns/jet_packed.py:43-53``)."""
    n, dim = x.shape
    nb = n - ni
    qi, qb = J.q(dim, 3), J.q(dim, boundary_order)
    inner = np.zeros((ni, qi, dim))
    inner[:, 0, :] = x[:ni]
    outer = np.zeros((nb, qb, dim))
    outer[:, 0, :] = x[ni:]
    for axis in range(dim):
        inner[:, J.unit(dim, axis), axis] = 1.0
        if boundary_order >= 1:
            outer[:, J.unit(dim, axis), axis] = 1.0
    return np.concatenate((inner.reshape(ni * qi, dim), outer.reshape(nb * qb, dim)))


def zero_rows(ni, nb, dim, boundary_order):
    qi, qb = J.q(dim, 3), J.q(dim, boundary_order)
    return np.concatenate((np.arange(ni) * qi, ni * qi + np.arange(nb) * qb)).astype(np.int64)


def _activation(z, ni, nb, dim, boundary_order):
    qi, qb = J.q(dim, 3), J.q(dim, boundary_order)
    c = z.shape[1]
    h = np.empty_like(z)
    aux = np.empty((ni + nb, c))
    if ni:
        part, a1 = J.tanh_jet(z[:ni * qi].reshape(ni, qi, c), dim, 3)
        h[:ni * qi] = part.reshape(ni * qi, c)
        aux[:ni] = a1
    if nb:
        part, a1 = J.tanh_jet(z[ni * qi:].reshape(nb, qb, c), dim, boundary_order)
        h[ni * qi:] = part.reshape(nb * qb, c)
        aux[ni:] = a1
    return h, aux


def _activation_vjp(h, aux, hbar, ni, nb, dim, boundary_order):
    qi, qb = J.q(dim, 3), J.q(dim, boundary_order)
    c = h.shape[1]
    out = np.empty_like(h)
    if ni:
        s = (ni, qi, c)
        out[:ni * qi] = J.tanh_vjp(h[:ni * qi].reshape(s), aux[:ni], hbar[:ni * qi].reshape(s),
                                   dim, 3).reshape(ni * qi, c)
    if nb:
        s = (nb, qb, c)
        out[ni * qi:] = J.tanh_vjp(h[ni * qi:].reshape(s), aux[ni:], hbar[ni * qi:].reshape(s),
                                   dim, boundary_order).reshape(nb * qb, c)
    return out


def evaluate(x, ni, pde_weights, boundary_weights, target, weights, biases, *,
             head="uvp", nu=0.07, gamma=0.2, bc=5.0, boundary_order=0, return_parts=False):
    """Return ``(loss, [dW_0..dW_L, db_0..db_L])`` as NumPy FP64."""
    x = np.asarray(x, dtype=np.float64)
    n, dim = x.shape
    nb = n - ni
    qi, qb = J.q(dim, 3), J.q(dim, boundary_order)
    zero = zero_rows(ni, nb, dim, boundary_order)
    h = coordinate_jets(x, ni, boundary_order)
    saved, auxs = [h], []
    for layer, (w, b) in enumerate(zip(weights, biases)):
        z = h @ np.asarray(w).T
        z[zero] += np.asarray(b)
        if layer + 1 < len(weights):
            h, a1 = _activation(z, ni, nb, dim, boundary_order)
            auxs.append(a1)
        else:
            h = z
        saved.append(h)
    y = saved[-1]
    cout = y.shape[1]
    li, si = RS.interior_seed(y[:ni * qi].reshape(ni, qi, cout), np.asarray(pde_weights), head, nu, gamma)
    lb, sb = RS.boundary_seed(y[ni * qi:].reshape(nb, qb, cout), np.asarray(boundary_weights),
                              np.asarray(target), bc, head, dim, boundary_order)
    loss = float(li.sum() + lb.sum())
    d = np.concatenate((si.reshape(ni * qi, cout), sb.reshape(nb * qb, cout)))
    dws, dbs = [None] * len(weights), [None] * len(weights)
    for layer in reversed(range(len(weights))):
        dws[layer] = d.T @ saved[layer]
        dbs[layer] = d[zero].sum(0)
        if layer:
            dh = d @ np.asarray(weights[layer])
            d = _activation_vjp(saved[layer], auxs[layer - 1], dh, ni, nb, dim, boundary_order)
    if return_parts:
        return loss, dws + dbs, {"outputs": y, "checkpoints": saved, "aux": auxs}
    return loss, dws + dbs


def evaluate_threaded(x, ni, pde_weights, boundary_weights, target, weights, biases, *,
                      threads, chunks=None, **options):
    """Same evaluation split over point chunks on ``threads`` host threads.

    Points are independent, so chunk losses and gradients add up to the full
    result (sum order differs; used for the timed CPU baseline).
    """
    x = np.asarray(x)
    nb = len(x) - ni
    chunks = chunks or threads
    ib = [ni * k // chunks for k in range(chunks + 1)]
    bb = [nb * k // chunks for k in range(chunks + 1)]
    pw, bw, tg = np.asarray(pde_weights), np.asarray(boundary_weights), np.asarray(target)

    def work(k):
        xi, xb = x[ib[k]:ib[k + 1]], x[ni + bb[k]:ni + bb[k + 1]]
        return evaluate(np.concatenate((xi, xb)), len(xi), pw[ib[k]:ib[k + 1]], bw[bb[k]:bb[k + 1]],
                        tg[bb[k]:bb[k + 1]], weights, biases, **options)

    with ThreadPoolExecutor(threads) as pool:
        results = list(pool.map(work, range(chunks)))
    loss = sum(r[0] for r in results)
    grads = [sum(r[1][i] for r in results) for i in range(len(results[0][1]))]
    return loss, grads

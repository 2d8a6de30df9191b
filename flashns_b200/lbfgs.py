"""Device-resident L-BFGS with a strong-Wolfe line search.

The vectors (parameters, gradients, the curvature history S, Y) stay on the GPU; each
iteration moves only O(history) numbers between host and device.

* Search direction: the compact representation of the L-BFGS inverse Hessian (Byrd,
  Nocedal and Schnabel, "Representations of quasi-Newton matrices and their use in
  limited memory methods", Math. Programming 63, 1994, Theorem 2.2) with H0 = gamma I:

      H g = gamma g + S cs + Y cy,   u = R^-1 (S^T g),
      cs = R^-T ((D + gamma Y^T Y) u - gamma Y^T g),   cy = -gamma u,

  where R is the upper triangle of S^T Y (oldest to newest) and D its diagonal.  The
  device computes S^T g and Y^T g (one block per dot product) and the combination; the
  host solves the two k x k triangular systems.
* Step length: strong Wolfe conditions (c1 = 1e-4, c2 = 0.9) by bracketing and zoom with
  cubic interpolation (Nocedal and Wright, Numerical Optimization, 2nd ed., Algorithms
  3.5 and 3.6, eq. 3.59).  Each trial sets x = x0 + t d on the device, replays the
  evaluation and reads back (f, g.d).
"""

import ctypes
import math

import numpy as np
import torch
from scipy.linalg import solve_triangular

from flashns_b200 import _lib


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


class DeviceLBFGS:
    """Minimize with ``evaluate()`` writing the loss into ``loss_view`` and the gradient
    into ``grad_view`` at the parameters currently in ``x`` (e.g. a CUDA-graph replay)."""

    def __init__(self, x, grad_view, loss_view, evaluate, *, history=50, c1=1e-4, c2=0.9, max_evals_per_search=25):
        self.x, self.g, self.f = x, grad_view, loss_view
        self.evaluate = evaluate
        self.n = x.numel()
        self.m, self.c1, self.c2, self.max_ls = history, c1, c2, max_evals_per_search
        dev = x.device
        z = lambda *shape: torch.zeros(*shape, dtype=torch.float64, device=dev)
        self.x0, self.g0, self.d = z(self.n), z(self.n), z(self.n)
        self.S, self.Y = z(self.m, self.n), z(self.m, self.n)
        self.dots = z(2 * self.m + 2)
        self.coef = z(2 * self.m)
        self.order_dev = torch.zeros(self.m, dtype=torch.int32, device=dev)
        self.host = torch.zeros(2 * self.m + 2, dtype=torch.float64).pin_memory()
        self.order = []  # physical rows, oldest first
        self.SY = np.zeros((self.m, self.m))  # SY[a, b] = s_a . y_b (a older than or equal to b)
        self.YY = np.zeros((self.m, self.m))
        self.evaluations = 0
        self.iterations = 0
        self.lib = _lib.library()
        self.stream = torch.cuda.current_stream(dev)
        self.fk = None

    # ---------------------------------------------------------------- device helpers
    def _s(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.x.device).cuda_stream)

    def _row_dots(self, rows, k, v, out):
        _lib.check(self.lib.flashns_b200_row_dots(_p(rows), self.n, k, _p(v), _p(out), self.n, self._s()), "row_dots")

    def _read(self, count):
        self.host[:count].copy_(self.dots[:count], non_blocking=True)
        torch.cuda.current_stream(self.x.device).synchronize()
        return self.host[:count].numpy().copy()

    def _phi(self, t):
        """Evaluate at x0 + t d; return (f, g.d)."""
        _lib.check(self.lib.flashns_b200_axpy(_p(self.x0), float(t), _p(self.d), _p(self.x), self.n, self._s()), "axpy")
        self.evaluate()
        self.evaluations += 1
        self._row_dots(self.g, 1, self.d, self.dots[1:])
        self.dots[0].copy_(self.f, non_blocking=True)
        f, gd = self._read(2)
        return float(f), float(gd)

    # ---------------------------------------------------------------- direction
    def _direction(self):
        k = len(self.order)
        if k == 0:
            self.d.copy_(self.g).neg_()
            return
        rows = self.order
        self._row_dots(self.S, k, self.g, self.dots)   # physical row r -> dots[r]
        self._row_dots(self.Y, k, self.g, self.dots[self.m:])
        h = self._read(2 * self.m)
        p1 = np.array([h[r] for r in rows])
        p2 = np.array([h[self.m + r] for r in rows])
        R = np.triu(self.SY[np.ix_(rows, rows)])
        D = np.diag(np.diag(R))
        YY = self.YY[np.ix_(rows, rows)]
        newest = rows[-1]
        gamma = self.SY[newest, newest] / self.YY[newest, newest]
        u = _solve_upper(R, p1)
        cs = _solve_lower(R.T, (D + gamma * YY) @ u - gamma * p2)
        cy = -gamma * u
        coef = torch.from_numpy(np.concatenate((cs, cy)))
        self.coef[:2 * k].copy_(coef.to(self.x.device, non_blocking=False))
        self.order_dev[:k].copy_(torch.tensor(rows, dtype=torch.int32))
        _lib.check(self.lib.flashns_b200_lbfgs_combine(_p(self.S), _p(self.Y), self.n, _p(self.order_dev), k,
                                                       _p(self.coef), _p(self.coef[k:]), _p(self.g), float(gamma),
                                                       _p(self.d), self.n, self._s()), "lbfgs_combine")

    def _push_pair(self):
        if len(self.order) == self.m:
            slot = self.order.pop(0)
        else:
            used = set(self.order)
            slot = next(r for r in range(self.m) if r not in used)
        _lib.check(self.lib.flashns_b200_lbfgs_pair(_p(self.x), _p(self.x0), _p(self.g), _p(self.g0),
                                                    _p(self.S[slot]), _p(self.Y[slot]), self.n, self._s()), "pair")
        rows = self.order + [slot]
        # s_a . y_new and y_a . y_new for every stored row a (physical indices 0..m-1 as used)
        self._row_dots(self.S, self.m, self.Y[slot], self.dots)
        self._row_dots(self.Y, self.m, self.Y[slot], self.dots[self.m:])
        h = self._read(2 * self.m)
        sy, yy = h[slot], h[self.m + slot]
        if not (sy > 1e-12 * max(yy, 1e-300)) or not math.isfinite(sy) or not math.isfinite(yy):
            return False  # curvature condition fails: the pair is not stored
        for a in rows:
            self.SY[a, slot] = h[a]
            self.YY[a, slot] = self.YY[slot, a] = h[self.m + a]
        self.order = rows
        return True

    # ---------------------------------------------------------------- line search
    def _line_search(self, f0, gd0, t):
        c1, c2 = self.c1, self.c2
        t_prev, f_prev, gd_prev = 0.0, f0, gd0
        best = (f0, 0.0, gd0)
        for i in range(self.max_ls):
            f, gd = self._phi(t)
            if f < best[0]:
                best = (f, t, gd)
            if f > f0 + c1 * t * gd0 or (i > 0 and f >= f_prev):
                return self._zoom(f0, gd0, t_prev, f_prev, gd_prev, t, f, gd, best, self.max_ls - i - 1)
            if abs(gd) <= -c2 * gd0:
                return t, f
            if gd >= 0:
                return self._zoom(f0, gd0, t, f, gd, t_prev, f_prev, gd_prev, best, self.max_ls - i - 1)
            t_prev, f_prev, gd_prev = t, f, gd
            t = min(2.0 * t, 1e10)
        return self._settle(best)

    def _zoom(self, f0, gd0, lo, f_lo, gd_lo, hi, f_hi, gd_hi, best, budget):
        c1, c2 = self.c1, self.c2
        for _ in range(max(budget, 0)):
            t = _cubic_min(lo, f_lo, gd_lo, hi, f_hi, gd_hi)
            a, b = min(lo, hi), max(lo, hi)
            if not (a + 0.1 * (b - a) <= t <= b - 0.1 * (b - a)):
                t = 0.5 * (a + b)
            f, gd = self._phi(t)
            if f < best[0]:
                best = (f, t, gd)
            if f > f0 + c1 * t * gd0 or f >= f_lo:
                hi, f_hi, gd_hi = t, f, gd
            else:
                if abs(gd) <= -c2 * gd0:
                    return t, f
                if gd * (hi - lo) >= 0:
                    hi, f_hi, gd_hi = lo, f_lo, gd_lo
                lo, f_lo, gd_lo = t, f, gd
            if abs(hi - lo) < 1e-16 * max(1.0, abs(lo)):
                break
        return self._settle(best)

    def _settle(self, best):
        """Budget exhausted: return to the best point seen (re-evaluated if needed)."""
        f, t, _ = best
        if t == 0.0:
            return 0.0, f
        self._phi(t)
        return t, f

    # ---------------------------------------------------------------- driver
    def step(self, iterations):
        """Run up to ``iterations`` iterations; return the current loss."""
        if self.fk is None:
            self.evaluate()
            self.evaluations += 1
            self.dots[0].copy_(self.f)
            self.fk = float(self._read(1)[0])
        for _ in range(iterations):
            self._direction()
            self._row_dots(self.g, 1, self.d, self.dots)
            gd0 = float(self._read(1)[0])
            if not gd0 < 0:  # not a descent direction: restart from steepest descent
                self.order = []
                self.d.copy_(self.g).neg_()
                self._row_dots(self.g, 1, self.d, self.dots)
                gd0 = float(self._read(1)[0])
                if not gd0 < 0:
                    break
            t0 = 1.0 if self.order else min(1.0, 1.0 / max(float(self.g.abs().sum()), 1e-300))
            self.x0.copy_(self.x)
            self.g0.copy_(self.g)
            t, f = self._line_search(self.fk, gd0, t0)
            if t == 0.0:  # no decrease along d: restore x0 (and its gradient) and stop
                self.x.copy_(self.x0)
                self.evaluate()
                self.evaluations += 1
                self.order = []
                break
            self._push_pair()
            self.fk = f
            self.iterations += 1
        return self.fk


def _solve_upper(R, b):
    return solve_triangular(R, b, lower=False, check_finite=False)


def _solve_lower(L, b):
    return solve_triangular(L, b, lower=True, check_finite=False)


def _cubic_min(x1, f1, g1, x2, f2, g2):
    """Minimizer of the cubic interpolating (f, f') at x1 and x2 (Nocedal-Wright eq. 3.59)."""
    d1 = g1 + g2 - 3.0 * (f1 - f2) / (x1 - x2) if x1 != x2 else float("nan")
    disc = d1 * d1 - g1 * g2
    if not (disc >= 0) or not math.isfinite(disc):
        return 0.5 * (x1 + x2)
    d2 = math.copysign(math.sqrt(disc), x2 - x1)
    den = g2 - g1 + 2.0 * d2
    if den == 0:
        return 0.5 * (x1 + x2)
    return x2 - (x2 - x1) * (g2 + d2 - d1) / den

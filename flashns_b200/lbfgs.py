"""Device-resident L-BFGS with a strong-Wolfe line search.

Everything of the quasi-Newton update lives on the GPU: the parameters, gradients, the
ring of curvature pairs (S, Y), their products S^T Y and Y^T Y, the pair count and the
coefficients.  One iteration launches a fixed sequence of small kernels (``csrc/lbfgs.cu``)
and reads back four scalars (f0, g0.d, f, g.d) once per line-search trial, so the common
iteration (first trial accepted) costs one evaluation and one host round trip.

* Search direction: the compact representation of the L-BFGS inverse Hessian (Byrd,
  Nocedal and Schnabel, "Representations of quasi-Newton matrices and their use in
  limited memory methods", Math. Programming 63, 1994, Theorem 2.2) with H0 = gamma I:

      H g = gamma g + S cs + Y cy,   u = R^-1 (S^T g),
      cs = R^-T ((D + gamma Y^T Y) u - gamma Y^T g),   cy = -gamma u,

  where R is the upper triangle of S^T Y (oldest to newest) and D its diagonal; the two
  triangular solves run in one CUDA block.  A new pair (s, y) is kept only when
  s.y > 1e-12 y.y; when the history is full the oldest pair drops out.
* Step length: strong Wolfe conditions (c1 = 1e-4, c2 = 0.9) by bracketing and zoom with
  cubic interpolation (Nocedal and Wright, Numerical Optimization, 2nd ed., Algorithms
  3.5 and 3.6, eq. 3.59).  Each trial sets x = x0 + t d on the device, runs the
  evaluation and reads back (f, g.d).
* Graph mode (``capture_evaluate`` given): the whole first trial of an iteration (pair
  update, direction, step, evaluation, read-back) and every further trial are two CUDA
  graphs; the host writes the step t and the pair flag into pinned memory that the graphs
  read, so an iteration is one graph launch and one synchronize.
"""

import ctypes
import math

import torch

from flashns_b200 import _lib

_GAMMA, _F0, _GD0, _F, _GD, _K, _T = range(7)
_MAX_HISTORY = 128


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


class DeviceLBFGS:
    """Minimize with ``evaluate()`` writing the loss into ``loss_view`` and the gradient
    into ``grad_view`` at the parameters currently in ``x`` (e.g. a CUDA-graph replay)."""

    def __init__(self, x, grad_view, loss_view, evaluate, *, history=50, c1=1e-4, c2=0.9, max_evals_per_search=25,
                 capture_evaluate=None):
        if not 1 <= history <= _MAX_HISTORY:
            raise ValueError(f"history must be in 1..{_MAX_HISTORY}")
        if x.dtype != torch.float64 or not x.is_cuda or not x.is_contiguous():
            raise ValueError("contiguous CUDA FP64 parameters required")
        self.x, self.g, self.f = x, grad_view, loss_view
        self.evaluate = evaluate
        self.n = x.numel()
        self.m, self.c1, self.c2, self.max_ls = history, c1, c2, max_evals_per_search
        self.slots = history + 1
        dev = x.device
        z = lambda *shape: torch.zeros(*shape, dtype=torch.float64, device=dev)
        self.x0, self.g0, self.d = z(self.n), z(self.n), z(self.n)
        self.S, self.Y = z(self.slots, self.n), z(self.slots, self.n)
        self.SY, self.YY = z(self.slots, self.slots), z(self.slots, self.slots)
        self.dots = z(2 * self.slots)
        self.coef = z(2 * _MAX_HISTORY)
        self.order = torch.zeros(_MAX_HISTORY, dtype=torch.int32, device=dev)
        self.state = torch.zeros(4, dtype=torch.int32, device=dev)  # k, spare slot, have_pair, 0
        self.scal = z(8)                                             # gamma, f0, g0.d, f, g.d, k
        self.host = torch.zeros(8, dtype=torch.float64).pin_memory()
        self.t_host = torch.zeros(1, dtype=torch.float64).pin_memory()
        self.flag_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.capture_evaluate = capture_evaluate  # records the evaluation kernels (graph mode)
        self.graphs = None
        self.evaluations = 0
        self.iterations = 0
        self.lib = _lib.library()
        self.fk = None

    # ---------------------------------------------------------------- device helpers
    def _s(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.x.device).cuda_stream)

    def _call(self, name, *args):
        _lib.check(getattr(self.lib, "flashns_b200_" + name)(*args, self._s()), name)

    def _read(self):
        self.host.copy_(self.scal, non_blocking=True)
        torch.cuda.current_stream(self.x.device).synchronize()
        return self.host.tolist()

    def _eval(self):
        self.evaluate()
        self.evaluations += 1

    def _trial_kernels(self, evaluate):
        """x = x0 + t d (t from scal), evaluation, scal[F] = f, scal[GD] = g.d."""
        self._call("lbfgs_step_point", _p(self.x0), _p(self.scal), _p(self.d), _p(self.x), self.n)
        evaluate()
        self.scal[_F:_F + 1].copy_(self.f.reshape(1))
        self._call("row_dots", _p(self.g), self.n, 1, _p(self.d), _p(self.scal[_GD:]), self.n)

    def _build_graphs(self):
        dev = self.x.device
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        first, trial = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(first, stream=stream):
            self.state[2:3].copy_(self.flag_host, non_blocking=True)
            self._direction(set_flag=False)
            self.scal[_T:_T + 1].copy_(self.t_host, non_blocking=True)
            self._trial_kernels(self.capture_evaluate)
            self.host.copy_(self.scal, non_blocking=True)
        with torch.cuda.graph(trial, stream=stream):
            self.scal[_T:_T + 1].copy_(self.t_host, non_blocking=True)
            self._trial_kernels(self.capture_evaluate)
            self.host.copy_(self.scal, non_blocking=True)
        torch.cuda.current_stream(dev).wait_stream(stream)
        self.graphs = (first, trial)

    def _replay(self, graph, t):
        self.t_host[0] = t
        graph.replay()
        self.evaluations += 1
        torch.cuda.current_stream(self.x.device).synchronize()
        h = self.host.tolist()
        return h[_F], h[_GD], h

    def _phi(self, t):
        """Evaluate at x0 + t d; return (f, g.d, the scalars read back)."""
        if self.graphs is not None:
            return self._replay(self.graphs[1], t)
        self.scal[_T:_T + 1].fill_(float(t))
        self._trial_kernels(self._eval)
        h = self._read()
        return h[_F], h[_GD], h

    def _first_trial(self, t, pair):
        """Direction (folding in the last pair when `pair`) and the trial at t."""
        if self.graphs is not None:
            self.flag_host[0] = int(pair)
            return self._replay(self.graphs[0], t)
        if pair:
            self.state[2:3].fill_(1)
        self._direction()
        return self._phi(t)

    # ---------------------------------------------------------------- direction
    def _direction(self, set_flag=True):
        """Fold the pair of the last accepted step into the history, then d = -H g; saves
        x0, g0, f0 and g0.d for the line search.  No host round trip."""
        slots = self.slots
        self._call("lbfgs_pair_slot", _p(self.x), _p(self.x0), _p(self.g), _p(self.g0), _p(self.S), _p(self.Y),
                   self.n, _p(self.state), self.n)
        self._call("lbfgs_ring_dots", _p(self.S), _p(self.Y), self.n, slots, None, _p(self.state), 1, _p(self.dots),
                   self.n)
        self._call("lbfgs_commit", _p(self.dots), _p(self.SY), _p(self.YY), slots, _p(self.state))
        if set_flag:
            self.state[2:3].zero_()
        self._call("lbfgs_ring_dots", _p(self.S), _p(self.Y), self.n, slots, _p(self.g), _p(self.state), 0,
                   _p(self.dots), self.n)
        self._call("lbfgs_coefficients", _p(self.SY), _p(self.YY), _p(self.dots), slots, _p(self.state),
                   _p(self.coef), _p(self.order), _p(self.scal))
        self._call("lbfgs_direction", _p(self.S), _p(self.Y), self.n, _p(self.order), _p(self.state), _p(self.coef),
                   _p(self.g), _p(self.scal), _p(self.d), self.n)
        self._call("lbfgs_save", _p(self.x), _p(self.g), _p(self.f), _p(self.x0), _p(self.g0), _p(self.scal), self.n)
        self._call("row_dots", _p(self.g), self.n, 1, _p(self.d), _p(self.scal[_GD0:]), self.n)

    def _restart(self):
        """Drop the history and return to x0 with its gradient and loss."""
        self.state.zero_()
        self.x.copy_(self.x0)
        self.g.copy_(self.g0)
        self.f.copy_(self.scal[_F0])

    # ---------------------------------------------------------------- line search
    def _line_search(self, f0, gd0, t, f, gd):
        """Strong Wolfe search; the trial at t is already evaluated as (f, gd)."""
        c1, c2 = self.c1, self.c2
        t_prev, f_prev, gd_prev = 0.0, f0, gd0
        best = (f0, 0.0, gd0)
        for i in range(self.max_ls):
            if i > 0:
                f, gd, _ = self._phi(t)
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
            f, gd, _ = self._phi(t)
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
        fresh = False
        if self.fk is None:
            self._eval()
            self.fk = float(self.f)
            self.pair = False
            fresh = True
            if self.capture_evaluate is not None and self.graphs is None:
                self._build_graphs()
        for _ in range(iterations):
            t0 = min(1.0, 1.0 / max(float(self.g.abs().sum()), 1e-300)) if fresh else 1.0
            f, gd, h = self._first_trial(t0, self.pair)
            gd0 = h[_GD0]
            if not gd0 < 0:  # not a descent direction: restart from steepest descent
                self._restart()
                t0 = min(1.0, 1.0 / max(float(self.g.abs().sum()), 1e-300))
                f, gd, h = self._first_trial(t0, False)
                gd0 = h[_GD0]
                if not gd0 < 0:
                    self._restart()
                    self.pair = False
                    break
            t, f = self._line_search(h[_F0], gd0, t0, f, gd)
            if t == 0.0:  # no decrease along d: back to x0 (and its gradient), drop the history
                self._restart()
                self.pair = False
                break
            self.pair = True  # the next direction folds in s = x - x0, y = g - g0
            self.fk = f
            fresh = False
            self.iterations += 1
        return self.fk


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

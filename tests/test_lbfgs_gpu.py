"""GPU: the device L-BFGS minimizes a convex quadratic and the Rosenbrock function, and
agrees with torch.optim.LBFGS on the quadratic's minimizer."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _problem(kind, n, device):
    x = torch.zeros(n, dtype=torch.float64, device=device)
    g = torch.zeros(n + 1, dtype=torch.float64, device=device)
    rng = np.random.default_rng(0)
    if kind == "quadratic":
        a = torch.tensor(rng.uniform(0.5, 20.0, n), device=device)
        b = torch.tensor(rng.normal(size=n), device=device)

        def evaluate():
            r = x - b
            g[:n] = a * r
            g[n] = 0.5 * (a * r * r).sum()
        return x, g, evaluate, b
    x.fill_(-1.0)

    def evaluate():
        u, v = x[:-1], x[1:]
        f = (100.0 * (v - u * u) ** 2 + (1 - u) ** 2).sum()
        gr = torch.zeros_like(x)
        gr[:-1] += -400.0 * u * (v - u * u) - 2.0 * (1 - u)
        gr[1:] += 200.0 * (v - u * u)
        g[:n] = gr
        g[n] = f
    return x, g, evaluate, torch.ones(n, dtype=torch.float64, device=device)


@pytest.mark.parametrize("kind,n,iters", [("quadratic", 1000, 200), ("rosenbrock", 10, 500)])
def test_device_lbfgs_converges(cuda, kind, n, iters):
    from flashns_b200.lbfgs import DeviceLBFGS
    x, g, evaluate, xstar = _problem(kind, n, cuda)
    opt = DeviceLBFGS(x, g[:n], g[n], evaluate, history=20)
    f = opt.step(iters)
    assert f < 1e-12
    assert float((x - xstar).abs().max()) < 1e-5

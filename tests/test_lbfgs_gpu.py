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


@pytest.mark.parametrize("graphs", [False, True])
@pytest.mark.parametrize("kind,n,iters", [("quadratic", 1000, 200), ("rosenbrock", 10, 500)])
def test_device_lbfgs_converges(cuda, kind, n, iters, graphs):
    """Eager launches and the two-graph mode (direction + trial captured once, replayed
    with the step and pair flag read from pinned memory) reach the minimizer."""
    from flashns_b200.lbfgs import DeviceLBFGS
    x, g, evaluate, xstar = _problem(kind, n, cuda)
    opt = DeviceLBFGS(x, g[:n], g[n], evaluate, history=20, capture_evaluate=evaluate if graphs else None)
    f = opt.step(iters)
    assert f < 1e-12
    assert float((x - xstar).abs().max()) < 1e-5


def test_adam_step_matches_reference_update(cuda):
    """flashns_b200_adam_step against the reference's FP64 Adam
    (experiments/pinn_solver/backends.py:216-240) written with torch ops."""
    import ctypes
    from flashns_b200 import _lib
    lib = _lib.library()
    gen = torch.Generator(device="cpu").manual_seed(4)
    n = 5000
    x = torch.randn(n, generator=gen, dtype=torch.float64).to(cuda)
    m, v = torch.zeros_like(x), torch.zeros_like(x)
    xr, mr, vr = x.clone(), m.clone(), v.clone()
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for step in range(1, 6):
        g = torch.randn(n, generator=gen, dtype=torch.float64).to(cuda)
        _lib.check(lib.flashns_b200_adam_step(p(x), p(g), p(m), p(v), n, 1e-3, 0.9, 0.999, 1e-8, step, s), "adam")
        mr.mul_(0.9).add_(g, alpha=0.1)
        vr.mul_(0.999).addcmul_(g, g, value=0.001)
        xr.sub_(1e-3 * (mr / (1 - 0.9 ** step)) / ((vr / (1 - 0.999 ** step)).sqrt() + 1e-8))
    torch.cuda.synchronize()
    assert float((x - xr).abs().max()) < 1e-14
    assert float((m - mr).abs().max()) < 1e-15 and float((v - vr).abs().max()) < 1e-15

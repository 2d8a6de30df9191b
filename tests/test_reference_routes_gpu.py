"""GPU: the reference's own GPU routes (its kernels compiled from its sources into
``baseline/_ref/`` by ``baseline/build_reference_gpu.py``) and this library's fused
evaluation agree on the same inputs, within the criterion the reference applies between
its own routes (``experiments/cuda_jet_h100/benchmark.py:151-158``,
``|a-b| <= 2e-12 + 2e-11|b|``).  Skipped when the reference kernels are not built."""

import pytest
import torch

from baseline.reference_routes import ROUTES, CapturedRoute, ReferenceKernels, available
from tests.cases import close_ratio, rel_norm

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not available(), reason="reference kernels not built (baseline/_ref)")]


def _setup(cuda, points, widths, seed=7510):
    from flashns_b200.evaluator import PackedEvaluator, flat_parameters
    from flashns_b200.ns_seed import NSLoss
    from flashns_b200.problems import reference_case, reference_parameters
    pts = reference_case(points, seed=seed)
    ws, bs = reference_parameters(widths, seed=seed)
    dev = lambda t: t.to(cuda).contiguous()
    x, pw, bw, target = dev(pts.x), dev(pts.pde_weights), dev(pts.boundary_weights), dev(pts.target)
    ev = PackedEvaluator(x, points, pw, bw, target, widths, head="uvp", boundary_order=0,
                         loss=NSLoss(viscosity=pts.viscosity, gradient_weight=0.2, boundary_weight=5.0), device=cuda)
    ours = ev(flat_parameters(ws, bs).to(cuda)).cpu()
    return (x, pw, bw, target, [dev(w) for w in ws], [dev(b) for b in bs], pts.viscosity), ours


@pytest.mark.parametrize("route", ROUTES)
@pytest.mark.parametrize("points,widths", [(600, [2, 64, 64, 3]), (257, [2, 32, 64, 3])])
def test_reference_route_matches_fused_evaluation(cuda, route, points, widths):
    (x, pw, bw, target, ws, bs, nu), ours = _setup(cuda, points, widths)
    captured = CapturedRoute(route, x, points, pw, bw, target, ws, bs, ReferenceKernels(), nu=nu, gamma=0.2)
    for _ in range(2):  # replays of one graph give the same result
        loss, grads = captured.replay()
        torch.cuda.synchronize()
        got = torch.cat([g.reshape(-1) for g in grads] + [loss.reshape(1)]).cpu()
        assert close_ratio(got.numpy(), ours.numpy()) <= 1, route
        assert rel_norm(got.numpy(), ours.numpy()) <= 1e-10


def test_reference_route_follows_new_inputs(cuda):
    """Static graph inputs refreshed in place (the e2e path of the benchmark arm)."""
    (x, pw, bw, target, ws, bs, nu), _ = _setup(cuda, 300, [2, 64, 64, 3])
    captured = CapturedRoute("v8", x, 300, pw, bw, target, ws, bs, ReferenceKernels(), nu=nu, gamma=0.2)
    (x2, _, _, _, ws2, bs2, _), ours2 = _setup(cuda, 300, [2, 64, 64, 3], seed=7600)
    for old, new in zip([x] + ws + bs, [x2] + ws2 + bs2):
        old.copy_(new)
    captured.refresh()
    loss, grads = captured.replay()
    got = torch.cat([g.reshape(-1) for g in grads] + [loss.reshape(1)]).cpu()
    assert close_ratio(got.numpy(), ours2.numpy()) <= 1


def test_reference_route_evaluator_for_the_solve(cuda):
    """The closure of the same-machine reference solve (baseline/reference_solve.py): the
    v8+ route with parameters as views of one flat vector writes the same [grad, loss] as
    this library's (u, v, p) evaluation of the Kovasznay point set."""
    from baseline.reference_solve import ReferenceRouteEvaluator
    from flashns_b200.evaluator import PackedEvaluator, flat_parameters, xavier_normal
    from flashns_b200.ns_seed import NSLoss
    from flashns_b200.problems import kovasznay
    pts = kovasznay(301, 77, seed=4, boundary_order=1)
    widths = [2, 64, 64, 3]
    loss = NSLoss(viscosity=pts.viscosity, gradient_weight=0.2, boundary_weight=5.0)
    ref = ReferenceRouteEvaluator(pts, widths, "uvp", 0, loss, cuda)
    ours = PackedEvaluator(pts.x, pts.interior_count, pts.pde_weights, pts.boundary_weights, pts.target, widths,
                           head="uvp", boundary_order=0, loss=loss, device=cuda)
    flat = flat_parameters(*xavier_normal(widths, 0)).to(cuda)
    out = torch.empty(ref.parameters + 1, dtype=torch.float64, device=cuda)
    ref(flat, out)
    expected = ours(flat)
    torch.cuda.synchronize()
    assert close_ratio(out.cpu().numpy(), expected.cpu().numpy()) <= 1

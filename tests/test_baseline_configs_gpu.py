"""GPU parity at the benchmark configurations' own sizes and widths, against the oracle.

The point counts here give every persistent CTA many tiles (at cfg1 about 15 half tiles
per CTA of the two-group kernels, each with its turn hand-over), which the small cases of
``test_eval_gpu.py`` do not reach:

* cfg0 in full: Kovasznay, 2,048 interior + 512 boundary points, 2-64x4-2 psi net;
* cfg1 in full: 16,384 + 4,096 points, the same net;
* cfg2's widths, 2-128x6-2, on 8,192 + 2,048 points;
* cfg3's widths, 3-128x5-2 with Q20 space-time jets and Taylor-Green targets, on
  4,096 + 1,024 points;
* the profile-only tgv64 net, 3-64x4-2 (the 3-D 64-wide kernels), on 4,096 + 1,024 points.

Points are uniform from seed 1, weights Xavier-normal from seed 0, boundary rows first
order, as in the benchmark.  Every value of ``[grad, loss]`` must meet the reference
criterion ``|a-b| <= 2e-12 + 2e-11|b|`` (sources/flashns_v8_reference/tests/verify_math.py:35-41)
and the whole vector the norm-wise relative error 1e-10 (the loss and parameter-gradient
tolerance of the path).  The CUDA path runs through the C ABI (``flashns_b200_eval``).
"""

import numpy as np
import pytest
import torch

from tests.cases import close_ratio, rel_norm

pytestmark = pytest.mark.gpu

CASES = {
    # name: (problem, interior, boundary, widths)
    "cfg0": ("kovasznay", 2048, 512, [2, 64, 64, 64, 64, 2]),
    "cfg1": ("kovasznay", 16384, 4096, [2, 64, 64, 64, 64, 2]),
    "cfg2_widths": ("kovasznay", 8192, 2048, [2] + [128] * 6 + [2]),
    "cfg3_widths": ("taylor_green", 4096, 1024, [3] + [128] * 5 + [2]),
    # the 3-D 64-wide kernels (fwd_head, bwd_fused on inner and first layers), which no
    # benchmark configuration reaches: tgv64's net
    "tgv64_widths": ("taylor_green", 4096, 1024, [3, 64, 64, 64, 64, 2]),
}


def problem(name):
    from flashns_b200.evaluator import xavier_normal
    from flashns_b200.problems import kovasznay, taylor_green
    kind, ni, nb, widths = CASES[name]
    build = kovasznay if kind == "kovasznay" else taylor_green
    pts = build(ni, nb, seed=1, boundary_order=1)
    ws, bs = xavier_normal(widths, 0)
    return pts, ws, bs, widths


def oracle_vector(pts, ws, bs):
    from oracle.evaluate import evaluate
    loss, grads = evaluate(pts.x.numpy(), pts.interior_count, pts.pde_weights.numpy(),
                           pts.boundary_weights.numpy(), pts.target.numpy(), [w.numpy() for w in ws],
                           [b.numpy() for b in bs], head="psi", nu=pts.viscosity, gamma=0.2, bc=5.0,
                           boundary_order=1)
    return np.concatenate([g.reshape(-1) for g in grads] + [[loss]])


@pytest.mark.parametrize("name", list(CASES))
def test_benchmark_configuration_matches_oracle(cuda, name):
    from flashns_b200.evaluator import PackedEvaluator, flat_parameters
    from flashns_b200.ns_seed import NSLoss
    pts, ws, bs, widths = problem(name)
    ev = PackedEvaluator(pts.x, pts.interior_count, pts.pde_weights, pts.boundary_weights, pts.target, widths,
                         head="psi", boundary_order=1,
                         loss=NSLoss(viscosity=pts.viscosity, gradient_weight=0.2, boundary_weight=5.0), device=cuda)
    out = ev(flat_parameters(ws, bs).to(cuda)).cpu().numpy()
    expected = oracle_vector(pts, ws, bs)
    ratio, rel = close_ratio(out, expected), rel_norm(out, expected)
    assert ratio <= 1.0, (name, ratio, rel)
    assert rel <= 1e-10, (name, ratio, rel)
    # the loss on its own, as the path's tolerance names it
    assert abs(out[-1] - expected[-1]) <= 1e-10 * abs(expected[-1]), (name, out[-1], expected[-1])

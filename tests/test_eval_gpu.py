"""Parity of the fused CUDA evaluation (through the C ABI) with the oracle and the
reference golden vectors."""

import numpy as np
import pytest
import torch

from tests.cases import close_ratio, flat, golden_pinn_cases, random_case, rel_norm

pytestmark = pytest.mark.gpu


def run(case, widths, head, order, loss, cuda):
    from flashns_b200.evaluator import PackedEvaluator
    t = lambda a: torch.tensor(a, dtype=torch.float64)
    ev = PackedEvaluator(t(case["x"]), case["ni"], t(case["pw"]), t(case["bw"]), t(case["target"]), widths,
                         head=head, boundary_order=order, loss=loss, device=cuda)
    out = ev(t(flat(case["ws"], case["bs"])).to(cuda))
    torch.cuda.synchronize()
    return ev, out.cpu().numpy()


def oracle(case, head, order, loss):
    from oracle.evaluate import evaluate
    value, grads = evaluate(case["x"], case["ni"], case["pw"], case["bw"], case["target"], case["ws"], case["bs"],
                            head=head, nu=loss.viscosity, gamma=loss.gradient_weight, bc=loss.boundary_weight,
                            boundary_order=order)
    return np.concatenate([g.reshape(-1) for g in grads] + [[value]])


@pytest.mark.parametrize("k", range(8))
def test_reference_golden_packed_pinn(cuda, k):
    from flashns_b200.ns_seed import NSLoss
    case = golden_pinn_cases()[k]
    loss = NSLoss(case["nu"], case["gamma"], case["bc"])
    _, out = run(case, case["widths"], "uvp", 0, loss, cuda)
    assert close_ratio(out[-1], case["loss"]) <= 1.0
    expected = np.concatenate([g.reshape(-1) for g in case["grads"]])
    assert close_ratio(out[:-1], expected) <= 1.0
    assert rel_norm(out[:-1], expected) <= 1e-10


CONFIGS = [
    # head, order, widths, ni, nb
    ("uvp", 0, (2, 64, 64, 64, 64, 3), 37, 11),
    ("uvp", 0, (2, 128, 128, 3), 21, 5),
    ("uvp", 0, (2, 20, 3), 9, 4),
    ("psi", 0, (2, 64, 64, 64, 64, 2), 37, 11),
    ("psi", 1, (2, 64, 64, 64, 64, 2), 37, 11),
    ("psi", 1, (2, 128, 128, 128, 2), 19, 29),
    ("psi", 1, (2, 100, 50, 2), 13, 7),
    ("psi", 0, (3, 128, 128, 2), 11, 13),
    ("psi", 1, (3, 128, 128, 128, 2), 11, 13),
    ("psi", 1, (3, 64, 64, 2), 17, 9),
    ("psi", 1, (3, 32, 2), 5, 3),
    ("psi", 1, (2, 64, 64, 2), 0, 9),
    ("psi", 1, (2, 64, 64, 2), 9, 0),
    ("uvp", 0, (2, 64, 64, 3), 1, 0),
    ("uvp", 0, (2, 64, 64, 3), 0, 1),
]


@pytest.mark.parametrize("head,order,widths,ni,nb", CONFIGS)
def test_against_oracle(cuda, head, order, widths, ni, nb):
    from flashns_b200.ns_seed import NSLoss
    loss = NSLoss(0.05, 0.2, 5.0)
    case = random_case(ni, nb, list(widths), head=head, boundary_order=order, seed=ni * 31 + nb)
    _, out = run(case, list(widths), head, order, loss, cuda)
    expected = oracle(case, head, order, loss)
    assert close_ratio(out, expected) <= 1.0, (close_ratio(out, expected), rel_norm(out, expected))


def test_empty_point_set(cuda):
    from flashns_b200.ns_seed import NSLoss
    case = random_case(0, 0, [2, 64, 64, 2], head="psi", boundary_order=1)
    _, out = run(case, [2, 64, 64, 2], "psi", 1, NSLoss(), cuda)
    assert np.all(out == 0.0)


def test_saturated_and_large_inputs(cuda):
    from flashns_b200.ns_seed import NSLoss
    case = random_case(23, 7, [2, 64, 64, 3], seed=5, scale=3.0)
    case["ws"][0] *= 12.0  # drives first-layer pre-activations deep into saturation
    loss = NSLoss()
    _, out = run(case, [2, 64, 64, 3], "uvp", 0, loss, cuda)
    expected = oracle(case, "uvp", 0, loss)
    assert close_ratio(out, expected) <= 1.0


def test_deterministic_and_stream_and_graph(cuda):
    from flashns_b200.ns_seed import NSLoss
    from flashns_b200.evaluator import PackedEvaluator
    widths = [2, 64, 64, 64, 2]
    case = random_case(613, 157, widths, head="psi", boundary_order=1, seed=9)
    t = lambda a: torch.tensor(a, dtype=torch.float64)
    ev = PackedEvaluator(t(case["x"]), case["ni"], t(case["pw"]), t(case["bw"]), t(case["target"]), widths,
                         head="psi", boundary_order=1, loss=NSLoss(0.05), device=cuda)
    params = t(flat(case["ws"], case["bs"])).to(cuda)
    a = ev(params).clone()
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        b = ev(params).clone()
    side.synchronize()
    assert torch.equal(a, b)
    out = torch.empty_like(a)
    with torch.cuda.stream(side):
        ev(params, out)  # warm-up on the capture stream
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            ev(params, out)
    for scale in (1.0, 0.5):
        params.mul_(scale)
        expect = ev(params).clone()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, expect)
    del graph


def test_point_linearity_at_scale(cuda):
    """loss and gradient are sums over points: two halves add up to the whole."""
    from flashns_b200.ns_seed import NSLoss
    from flashns_b200.evaluator import PackedEvaluator
    widths = [2, 64, 64, 64, 64, 2]
    case = random_case(16384, 4096, widths, head="psi", boundary_order=1, seed=3, scale=0.6)
    t = lambda a: torch.tensor(a, dtype=torch.float64)
    params = t(flat(case["ws"], case["bs"])).to(cuda)
    x, ni = case["x"], case["ni"]
    full = PackedEvaluator(t(x), ni, t(case["pw"]), t(case["bw"]), t(case["target"]), widths,
                           head="psi", boundary_order=1, loss=NSLoss(0.05), device=cuda)(params)
    h, hb = ni // 2, 4096 // 2
    parts = []
    for si, sb in ((slice(0, h), slice(0, hb)), (slice(h, ni), slice(hb, 4096))):
        xs = np.concatenate((x[:ni][si], x[ni:][sb]))
        nis = si.stop - si.start
        parts.append(PackedEvaluator(t(xs), nis, t(case["pw"][si]), t(case["bw"][sb]), t(case["target"][sb]), widths,
                                     head="psi", boundary_order=1, loss=NSLoss(0.05), device=cuda)(params))
    total = (parts[0] + parts[1]).cpu().numpy()
    assert rel_norm(total, full.cpu().numpy()) <= 1e-12

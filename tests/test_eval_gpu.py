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
    assert rel_norm(out, expected) <= 1e-10, rel_norm(out, expected)


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


@pytest.mark.parametrize("dim,order", [(2, 1), (2, 0), (3, 1)])
def test_field_evaluator_matches_oracle(cuda, dim, order):
    from flashns_b200.evaluator import FieldEvaluator
    from oracle import residuals as RS
    from oracle.evaluate import evaluate
    widths = [dim, 64, 64, 2]
    case = random_case(0, 57, widths, head="psi", boundary_order=order, seed=11)
    fe = FieldEvaluator(torch.tensor(case["x"]), widths, head="psi", boundary_order=order, device=cuda)
    got = fe(torch.tensor(flat(case["ws"], case["bs"])).to(cuda)).cpu().numpy()
    _, _, parts = evaluate(case["x"], 0, case["pw"], case["bw"], case["target"], case["ws"], case["bs"], head="psi",
                           boundary_order=order, return_parts=True)
    qb = dim + 1 if order else 1
    rows = parts["outputs"].reshape(57, qb, 2)
    expect = RS.boundary_fields(rows, "psi", dim, order)
    assert close_ratio(got, expect) <= 1.0


def test_solver_runs_and_reduces_loss(cuda):
    """A short solve on a small point set: the machinery (graph-captured closure, L-BFGS,
    acceptance on a small grid) runs and the loss decreases."""
    from flashns_b200.solver import solve
    log = []
    r = solve(interior=512, boundary=128, widths=(2, 32, 32, 2), max_iterations=40, check_every=20, grid=21, adam_steps=50,
              device=cuda, log=log.append)
    assert r["iterations"] >= 20 and r["evaluations"] >= 20
    first = __import__("json").loads(log[0])["loss"]
    assert r["final_loss"] < first


def test_solver_uvp_head_runs_and_reduces_loss(cuda):
    """The (u, v, p) head of the solver (the reference's objective, value boundary rows):
    the captured closure, L-BFGS and the acceptance fields run and the loss decreases."""
    from flashns_b200.solver import solve
    log = []
    r = solve(interior=512, boundary=128, widths=(2, 32, 32, 3), max_iterations=40, check_every=20, grid=21,
              adam_steps=50, device=cuda, log=log.append, head="uvp")
    assert r["head"] == "uvp" and r["iterations"] >= 20
    first = __import__("json").loads(log[0])["loss"]
    assert r["final_loss"] < first


@pytest.mark.gpu
def test_bounded_wait_reports_instead_of_hanging(cuda):
    """An mbarrier that nothing arrives at: the kernel's bounded wait gives up, raises the
    device fault word and returns, and the context stays usable; normal evaluations leave
    the word clear."""
    import ctypes
    from flashns_b200 import _lib
    lib = _lib.library()
    fault = ctypes.c_int(-1)
    _lib.check(lib.flashns_b200_device_fault(ctypes.byref(fault), 1), "device_fault")
    from flashns_b200.ns_seed import NSLoss
    widths = [2, 64, 64, 64, 2]
    case = random_case(64, 16, widths, head="psi", boundary_order=1, seed=3)
    loss = NSLoss(0.05, 0.0, 2.0)
    run(case, widths, "psi", 1, loss, cuda)
    torch.cuda.synchronize()
    _lib.check(lib.flashns_b200_device_fault(ctypes.byref(fault), 0), "device_fault")
    assert fault.value == 0
    gave_up = torch.full((1,), -1, dtype=torch.int32, device=cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.flashns_b200_wait_selftest(200, ctypes.c_void_p(gave_up.data_ptr()), stream), "wait_selftest")
    torch.cuda.synchronize()
    assert int(gave_up.item()) == 1
    _lib.check(lib.flashns_b200_device_fault(ctypes.byref(fault), 1), "device_fault")
    assert fault.value == 1
    _lib.check(lib.flashns_b200_device_fault(ctypes.byref(fault), 0), "device_fault")
    assert fault.value == 0
    _, out = run(case, widths, "psi", 1, loss, cuda)  # the context still works
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out, oracle(case, "psi", 1, loss), rtol=1e-9, atol=1e-12)


@pytest.mark.gpu
def test_unaligned_parameter_view(cuda):
    """A parameter view off a 16-byte boundary evaluates like the aligned vector (the C ABI
    reads parameters in place when no width needs padding, so the binding realigns)."""
    from flashns_b200.ns_seed import NSLoss
    widths = [2, 64, 64, 2]
    case = random_case(40, 12, widths, head="psi", boundary_order=1, seed=5)
    loss = NSLoss(0.05, 0.0, 2.0)
    ev, ref = run(case, widths, "psi", 1, loss, cuda)
    p = torch.tensor(flat(case["ws"], case["bs"]), dtype=torch.float64)
    buf = torch.zeros(p.numel() + 1, dtype=torch.float64, device=cuda)
    view = buf[1:]
    view.copy_(p)
    assert view.data_ptr() % 16 != 0
    out = ev(view)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_input_arena_single_copy_refreshes_every_input(cuda):
    """PackedEvaluator.input_arena: the inputs become views of one device buffer, results
    are unchanged, and one host-to-device copy of new host values is what the next
    evaluation sees."""
    import torch
    from flashns_b200.evaluator import PackedEvaluator, flat_parameters, xavier_normal
    from flashns_b200.ns_seed import NSLoss
    from flashns_b200.problems import kovasznay
    widths = [2, 64, 64, 64, 2]
    a, b = kovasznay(301, 77, seed=11), kovasznay(301, 77, seed=12)
    make = lambda pts: PackedEvaluator(pts.x, pts.interior_count, pts.pde_weights, pts.boundary_weights, pts.target,
                                       widths, head="psi", boundary_order=1, loss=NSLoss(0.05, 0.0, 5.0), device=cuda)
    ev, ev_b = make(a), make(b)
    ws, bs = xavier_normal(widths, 0)
    p = flat_parameters(ws, bs)
    before = ev(p.to(cuda)).cpu()
    host, device, dparams = ev.input_arena(p)
    assert host.is_pinned() and device.is_cuda and dparams.data_ptr() % 16 == 0
    assert ev.x.data_ptr() == device.data_ptr()
    assert torch.equal(ev(dparams).cpu(), before)
    # stage point set b and new parameters on the host, then one copy
    p2 = p * 0.9
    n = [a.x.numel(), a.pde_weights.numel(), a.boundary_weights.numel(), a.target.numel()]
    o = 0
    for t, k in zip([b.x, b.pde_weights, b.boundary_weights, b.target], n):
        host[o:o + k] = t.reshape(-1)
        o += k + (k & 1)
    host[o:o + p2.numel()] = p2
    device.copy_(host)
    assert torch.equal(ev(dparams).cpu(), ev_b(p2.to(cuda)).cpu())

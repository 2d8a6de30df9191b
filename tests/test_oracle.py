"""CPU: the oracle against the reference golden vectors and against nested autograd."""

import numpy as np
import pytest

from tests.cases import GOLDEN, close_ratio, golden_pinn_cases, random_case

from oracle import jets as J
from oracle import residuals as RS
from oracle.evaluate import _activation, _activation_vjp, evaluate
from oracle.nested_ad import nested_step


@pytest.mark.parametrize("k", range(8))
def test_oracle_matches_reference_packed_pinn(k):
    case = golden_pinn_cases()[k]
    loss, grads = evaluate(case["x"], case["ni"], case["pw"], case["bw"], case["target"], case["ws"], case["bs"],
                           head="uvp", nu=case["nu"], gamma=case["gamma"], bc=case["bc"])
    assert close_ratio(loss, case["loss"]) <= 1.0
    for a, b in zip(grads, case["grads"]):
        assert close_ratio(a, b) <= 1.0


def test_reference_packed_pinn_agrees_with_reference_nested_ad():
    g = np.load(GOLDEN / "reference_packed_pinn.npz")
    checked = 0
    for k in range(int(g["pinn_count"])):
        p = f"pinn{k}_"
        if p + "nested_loss" not in g:
            continue
        assert close_ratio(g[p + "loss"], g[p + "nested_loss"]) <= 1.0
        n = len(g[p + "widths"]) - 1
        for i in range(2 * n):
            assert close_ratio(g[p + f"g{i}"], g[p + f"nested_g{i}"]) <= 1.0
        checked += 1
    assert checked >= 4


def test_oracle_activation_matches_reference():
    a = np.load(GOLDEN / "reference_activation.npz")
    for k in range(int(a["act_count"])):
        p = f"act{k}_"
        dim, full, value = (int(v) for v in a[p + "meta"])
        h, aux = _activation(a[p + "z"], full, value, dim, 0)
        dz = _activation_vjp(h, aux, a[p + "seed"], full, value, dim, 0)
        assert close_ratio(h, a[p + "h"]) <= 1.0
        assert close_ratio(aux, a[p + "a1"]) <= 1.0
        assert close_ratio(dz, a[p + "dz"]) <= 1.0


def test_oracle_seed_matches_reference():
    s = np.load(GOLDEN / "reference_seed.npz")
    for k in range(int(s["seed_count"])):
        p = f"seed{k}_"
        nu, gamma = (float(v) for v in s[p + "nu_gamma"])
        loss, seed = RS.interior_seed(s[p + "jets"], s[p + "w"], "uvp", nu, gamma)
        assert close_ratio(loss.sum(), s[p + "loss"]) <= 1.0
        assert close_ratio(seed, s[p + "seed"]) <= 1.0
        assert close_ratio(RS.residual_values(s[p + "jets"], "uvp", nu, gamma), s[p + "res"]) <= 1.0


NESTED = [
    ("uvp", 0, (2, 7, 6, 3), 5, 3),
    ("psi", 0, (2, 7, 6, 2), 5, 3),
    ("psi", 1, (2, 7, 6, 2), 5, 3),
    ("psi", 1, (3, 7, 6, 2), 5, 3),
    ("psi", 0, (3, 5, 4, 2), 4, 2),
    ("psi", 1, (2, 9, 2), 1, 0),
    ("psi", 1, (3, 9, 2), 0, 2),
]


@pytest.mark.parametrize("head,order,widths,ni,nb", NESTED)
def test_oracle_matches_nested_autograd(head, order, widths, ni, nb):
    """Pins the stream-function heads, which have no reference counterpart."""
    case = random_case(ni, nb, list(widths), head=head, boundary_order=order, seed=ni + 7 * nb)
    opts = dict(head=head, nu=0.05, gamma=0.2, bc=5.0, boundary_order=order)
    a = evaluate(case["x"], ni, case["pw"], case["bw"], case["target"], case["ws"], case["bs"], **opts)
    b = nested_step(case["x"], ni, case["pw"], case["bw"], case["target"], case["ws"], case["bs"], **opts)
    assert close_ratio(a[0], b[0]) <= 1.0
    for x, y in zip(a[1], b[1]):
        assert close_ratio(x, y) <= 1.0


def test_truncated_basis_is_a_prefix():
    for dim in (2, 3):
        assert J.basis(dim, 1) == J.basis(dim, 3)[:dim + 1]
        assert J.basis(dim, 0) == ((0,) * dim,)
        assert J.q(dim) == (10 if dim == 2 else 20)


def test_kovasznay_and_tgv_fields_solve_the_equations():
    """Analytic stream functions of the configs give zero psi-head residuals."""
    import math
    import torch
    re = 20.0
    nu = 1.0 / re
    lam = re / 2 - math.sqrt(re * re / 4 + 4 * math.pi ** 2)
    x = torch.tensor(np.random.default_rng(0).uniform(-0.5, 1.0, size=(64, 2)), dtype=torch.float64, requires_grad=True)

    def grad(y):
        return torch.autograd.grad(y.sum(), x, create_graph=True)[0]

    psi = x[:, 1] - torch.exp(lam * x[:, 0]) * torch.sin(2 * math.pi * x[:, 1]) / (2 * math.pi)
    p = 0.5 * (1 - torch.exp(2 * lam * x[:, 0]))
    gp, gpp = grad(psi), grad(p)
    u, v = gp[:, 1], -gp[:, 0]
    gu, gv = grad(u), grad(v)
    ru = u * gu[:, 0] + v * gu[:, 1] + gpp[:, 0] - nu * (grad(gu[:, 0])[:, 0] + grad(gu[:, 1])[:, 1])
    rv = u * gv[:, 0] + v * gv[:, 1] + gpp[:, 1] - nu * (grad(gv[:, 0])[:, 0] + grad(gv[:, 1])[:, 1])
    assert float(ru.detach().abs().max()) < 1e-12 and float(rv.detach().abs().max()) < 1e-12
    expect_u = 1 - torch.exp(lam * x[:, 0]) * torch.cos(2 * math.pi * x[:, 1])
    assert float((u - expect_u).detach().abs().max()) < 1e-13


@pytest.mark.parametrize("dim", [2, 3])
def test_oracle_tanh_jet_tails_vs_100_digit_reference(dim):
    """Saturated centers up to 350: every jet coefficient of the oracle's stable tanh
    matches 100-digit mpmath (criterion of the reference's tests/test_jet_stable.py:28-42)."""
    from oracle import jets as J
    from tests.tails import expected_jets, input_jets, within_tail_tolerance
    h, a1 = J.tanh_jet(input_jets(dim), dim)
    ok = within_tail_tolerance(h, expected_jets(dim))
    assert ok.all(), np.argwhere(~ok)


@pytest.mark.parametrize("center", [0.0, 5.0, 20.0, -20.0, 100.0, 350.0])
def test_stable_tanh_nested_derivatives_vs_100_digit_reference(center):
    """flashns_b200.jet_stable.stable_tanh: four nested autograd derivatives against mpmath
    (the reference's tests/test_jet_stable.py:28-42 on this library's helper)."""
    import torch

    from flashns_b200.jet_stable import stable_tanh
    from tests.tails import tanh_derivative, within_tail_tolerance
    x = torch.tensor(center, dtype=torch.float64, requires_grad=True)
    derivative = stable_tanh(x)
    for order in range(1, 5):
        (derivative,) = torch.autograd.grad(derivative, x, create_graph=True)
        assert within_tail_tolerance(float(derivative.detach()), tanh_derivative(center, order)), (center, order)


def test_oracle_fourth_derivative_vjp_vs_100_digit_reference():
    """The VJP of the x^3 coefficient at z0 needs tanh'''' (the reference's
    sources/flashns_v8_reference/tests/verify_math.py:127-139)."""
    from oracle import jets as J
    from tests.tails import fourth_derivative_case
    z, seed, expected = fourth_derivative_case()
    h, a1 = J.tanh_jet(z, 2)
    got = J.tanh_vjp(h, a1, seed, 2)[:, 0, 0]
    assert np.all(np.abs(got - expected) <= 1e-30 + 2e-12 * np.abs(expected)), (got, expected)


def test_oracle_a1_tails_vs_420_digit_reference():
    """a1 = sech^2 z0 from r = exp(-|z0|) into the subnormal range, and the information it
    keeps where tanh rounds to 1 (verify_math.py:181-209)."""
    from oracle import jets as J
    from tests.tails import A1_PROBES, a1_tail_ok
    for z in A1_PROBES:
        for s in (1.0, -1.0):
            assert a1_tail_ok(J.stable_a1(np.array(s * z)), s * z), s * z
    assert np.tanh(20.0) == np.tanh(21.0) == 1.0
    assert J.stable_a1(np.array(20.0)) != J.stable_a1(np.array(21.0))

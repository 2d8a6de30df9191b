"""CPU: the orchestration of the reference's GPU routes (``baseline/reference_routes.py``).

The routes run here on CPU tensors with the reference kernels' contracts computed by the
oracle (``OracleKernels``), so what is checked is the restated orchestration around the
kernels: the packed v8 routes (with and without the opt-in fused hooks) against the
golden outputs of the reference's own ``PackedPINN``, the dense F / B1 routes against the oracle evaluation, and the torch
residual used for the dense routes' autograd seed against the oracle residual.
"""

import numpy as np
import pytest
import torch

from baseline.reference_routes import (coordinate_jets, dense_step, packed_coordinates, packed_step,
                                       uvp_residual_per_point, zero_rows)
from oracle import jets as J
from oracle.evaluate import evaluate
from oracle.residuals import interior_seed
from tests.cases import close_ratio, golden_pinn_cases, random_case


def _np(t):
    return t.detach().numpy()


class OracleKernels:
    """The reference kernels' input/output contracts (stable_kernels.cu, stable_dgrad.cu,
    native.cu) evaluated by the CPU oracle."""

    def forward(self, z, dim):
        h, a1 = J.tanh_jet(_np(z), dim)
        return torch.from_numpy(h), torch.from_numpy(a1)

    def vjp(self, h, a1, hbar, dim):
        return torch.from_numpy(J.tanh_vjp(_np(h), _np(a1), _np(hbar), dim))

    def dgrad(self, d, w, h, a1, dim, backend):
        assert backend in ("F", "B1")
        return self.vjp(h, a1, d @ w, dim)

    def packed_forward(self, full, value, dim, z):
        q, c = J.q(dim), z.shape[1]
        hf, af = J.tanh_jet(_np(z[:full * q]).reshape(full, q, c), dim)
        hv, av = J.tanh_jet(_np(z[full * q:])[:, None, :], dim)
        return (torch.from_numpy(np.concatenate((hf.reshape(full * q, c), hv[:, 0]))),
                torch.from_numpy(np.concatenate((af, av))))

    def packed_vjp(self, full, value, dim, h, a1, hbar):
        q = J.q(dim)
        c = h.shape[1]
        zf = J.tanh_vjp(_np(h[:full * q]).reshape(full, q, c), _np(a1[:full]),
                        _np(hbar[:full * q]).reshape(full, q, c), dim)
        zv = _np(hbar[full * q:]) * _np(a1[full:])
        return torch.from_numpy(np.concatenate((zf.reshape(full * q, c), zv)))

    def first_affine_activation(self, full, value, dim, x, w, b):
        z = packed_coordinates(x, full) @ w.T
        z[zero_rows(full, value, J.q(dim), x.device)] += b
        return self.packed_forward(full, value, dim, z)

    def first_activation_wgrad(self, full, value, dim, x, h, a1, hbar):
        zbar = self.packed_vjp(full, value, dim, h, a1, hbar)
        return zbar.T @ packed_coordinates(x, full), zbar[zero_rows(full, value, J.q(dim), x.device)].sum(0)

    def tail3(self, full, value, dim, d, w, h, a1):
        return self.packed_vjp(full, value, dim, h, a1, d @ w)

    def seed(self, jets, boundary, pde_weights, boundary_weights, target, nu, gamma, bc):
        per_point, di = interior_seed(_np(jets), _np(pde_weights), "uvp", nu, gamma)
        err = _np(boundary) - _np(target)
        total = per_point.sum() + bc * (_np(boundary_weights) * err * err).sum()
        return torch.tensor(total), torch.from_numpy(di), torch.from_numpy(2.0 * bc * _np(boundary_weights) * err)


def T(a):
    return torch.tensor(np.asarray(a), dtype=torch.float64)


def test_coordinate_jets_match_the_packed_layout():
    x = T(np.random.default_rng(3).normal(size=(7, 2)))
    dense = coordinate_jets(x)
    assert torch.equal(dense[:, 0], x)
    assert torch.equal(dense[:, J.unit(2, 0), 0], torch.ones(7, dtype=torch.float64))
    assert torch.equal(dense[:, J.unit(2, 1), 1], torch.ones(7, dtype=torch.float64))
    rest = dense[:, 1:]
    assert int((rest != 0).sum()) == 14 and float(rest.sum()) == 14.0  # nothing else is set
    packed = packed_coordinates(x, 4)
    assert packed.shape == (4 * 10 + 3, 2)
    assert torch.equal(packed[:40], dense[:4].reshape(40, 2)) and torch.equal(packed[40:], x[4:])


@pytest.mark.parametrize("nu,gamma", [(0.07, 0.2), (0.05, 0.0), (0.01, 1.3)])
def test_torch_residual_matches_oracle(nu, gamma):
    rng = np.random.default_rng(41)
    jets = rng.normal(size=(33, 10, 3))
    expected, _ = interior_seed(jets, np.ones(33), "uvp", nu, gamma)
    assert close_ratio(_np(uvp_residual_per_point(T(jets), nu, gamma)), expected) <= 1


def test_torch_residual_seed_is_the_oracle_seed():
    rng = np.random.default_rng(42)
    jets, w = rng.normal(size=(19, 10, 3)), rng.uniform(0, 1, size=19)
    leaf = T(jets).requires_grad_()
    (T(w) * uvp_residual_per_point(leaf, 0.07, 0.2)).sum().backward()
    _, seed = interior_seed(jets, w, "uvp", 0.07, 0.2)
    assert close_ratio(_np(leaf.grad), seed) <= 1


@pytest.mark.parametrize("hooks", [False, True])
def test_v8_routes_reproduce_reference_packed_pinn(hooks):
    for c in golden_pinn_cases():
        total, grads = packed_step(T(c["x"]), c["ni"], T(c["pw"]), T(c["bw"]), T(c["target"]),
                                   [T(w) for w in c["ws"]], [T(b) for b in c["bs"]], OracleKernels(),
                                   nu=c["nu"], gamma=c["gamma"], bc=c["bc"], hooks=hooks)
        assert close_ratio(float(total), c["loss"]) <= 1, c["name"]
        assert len(grads) == len(c["grads"])
        for got, exp in zip(grads, c["grads"]):
            assert close_ratio(_np(got), exp) <= 1, c["name"]


@pytest.mark.parametrize("backend", ["F", "B1"])
@pytest.mark.parametrize("widths", [[2, 16, 16, 3], [2, 24, 3], [2, 8, 12, 10, 3]])
def test_dense_routes_match_oracle(backend, widths):
    c = random_case(23, 0, widths, seed=7)
    ws, bs = [T(w) for w in c["ws"]], [T(b) for b in c["bs"]]
    total, grads = dense_step(T(c["x"]), T(c["pw"]), 1.0, ws, bs, OracleKernels(), backend, nu=0.07, gamma=0.2)
    ref_loss, ref_grads = evaluate(c["x"], 23, c["pw"], np.zeros((0, 3)), np.zeros((0, 3)), c["ws"], c["bs"],
                                   head="uvp", nu=0.07, gamma=0.2)
    assert close_ratio(float(total), ref_loss) <= 1
    for got, exp in zip(grads, ref_grads):
        assert close_ratio(_np(got), exp) <= 1


def test_dense_route_quadrature_over_denominator():
    """quadrature / denominator weighting equals globally normalized weights."""
    c = random_case(12, 0, [2, 10, 3], seed=9)
    ws, bs = [T(w) for w in c["ws"]], [T(b) for b in c["bs"]]
    q = np.full(12, 1.0)
    a = dense_step(T(c["x"]), T(q), 12.0, ws, bs, OracleKernels(), "F")
    b = dense_step(T(c["x"]), T(q / 12.0), 1.0, ws, bs, OracleKernels(), "F")
    assert close_ratio(float(a[0]), float(b[0])) <= 1
    for g, h in zip(a[1], b[1]):
        assert close_ratio(_np(g), _np(h)) <= 1

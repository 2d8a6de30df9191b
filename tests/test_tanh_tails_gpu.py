"""GPU: the stable tanh jet kernels at saturated centers (up to |z0| = 350) against
100-digit mpmath, with the reference's tail criterion |a - e| <= 1e-11 |e| + 8 ulp(e)
(tests/test_jet_stable.py:28-42 of the reference).  The fused evaluation kernels use the
same generated jet functions as these entry points (``jets_generated.cuh``)."""

import math

import numpy as np
import pytest
import torch

from tests.tails import CENTERS, expected_jets, input_jets, tanh_derivative, within_tail_tolerance

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dim", [2, 3])
def test_dense_activation_tails(cuda, dim):
    from flashns_b200.native import Native
    z = torch.tensor(input_jets(dim), dtype=torch.float64, device=cuda)
    h, a1 = Native().forward(z, dim)
    ok = within_tail_tolerance(h.cpu().numpy(), expected_jets(dim))
    assert ok.all(), np.argwhere(~ok)
    sech2 = np.array([[tanh_derivative(c, 1)] for c in CENTERS])
    assert within_tail_tolerance(a1.cpu().numpy(), sech2).all()


@pytest.mark.parametrize("dim", [2, 3])
def test_packed_activation_tails(cuda, dim):
    """Full-jet rows and value rows of the packed layout (flashns_v8_activation)."""
    from flashns_b200.jet_packed import PackedLayout
    from flashns_b200.native import NativeCUDA
    full = input_jets(dim)
    q = full.shape[1]
    rows = np.concatenate((full.reshape(len(CENTERS) * q, 1), np.array(CENTERS)[:, None]))
    layout = PackedLayout(len(CENTERS), len(CENTERS), dim)
    h, a1 = NativeCUDA().activation_factory(layout).forward(torch.tensor(rows, dtype=torch.float64, device=cuda))
    h, a1 = h.cpu().numpy(), a1.cpu().numpy()
    ok = within_tail_tolerance(h[:len(CENTERS) * q].reshape(full.shape), expected_jets(dim))
    assert ok.all(), np.argwhere(~ok)
    values = np.array([[math.tanh(c)] for c in CENTERS])
    assert within_tail_tolerance(h[len(CENTERS) * q:], values).all()
    sech2 = np.array([[tanh_derivative(c, 1)] for c in CENTERS] * 2)
    assert within_tail_tolerance(a1, sech2).all()


def test_fourth_derivative_vjp(cuda):
    """The VJP kernel at z0 for a seed on the x^3 coefficient: tanh''''(z0)/6
    (the reference's sources/flashns_v8_reference/tests/verify_math.py:127-139)."""
    from flashns_b200.native import Native
    from tests.tails import fourth_derivative_case
    z, seed, expected = fourth_derivative_case()
    nat = Native()
    h, a1 = nat.forward(torch.tensor(z, dtype=torch.float64, device=cuda), 2)
    got = nat.vjp(h, a1, torch.tensor(seed, dtype=torch.float64, device=cuda), 2)[:, 0, 0].cpu().numpy()
    assert np.all(np.abs(got - expected) <= 1e-30 + 2e-12 * np.abs(expected)), (got, expected)


def test_a1_tails(cuda):
    """a1 = sech^2 z0 into the subnormal range against 420-digit mpmath: relative 5e-13
    where it is a normal double.  Below that the GPU's exp may round one ulp away from
    the host's, so the absolute bound is 4 subnormal quanta (the reference allows its
    CPU 2); and a1 still separates z0 = 20 from 21, where tanh rounds both to 1."""
    from flashns_b200.native import Native
    from tests.tails import A1_PROBES, a1_tail_ok
    zs = [s * z for z in A1_PROBES for s in (1.0, -1.0)]
    z = torch.zeros(len(zs), 10, 1, dtype=torch.float64)
    z[:, 0, 0] = torch.tensor(zs, dtype=torch.float64)
    h, a1 = Native().forward(z.to(cuda), 2)
    a1 = a1[:, 0].cpu().numpy()
    for value, z0 in zip(a1, zs):
        assert a1_tail_ok(value, z0, quanta=4), z0
    i20, i21 = zs.index(20.0), zs.index(21.0)
    assert float(h[i20, 0, 0]) == float(h[i21, 0, 0]) == 1.0 and a1[i20] != a1[i21]

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

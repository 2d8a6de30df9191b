"""GPU: NaN and Inf propagation of the coordinate weight-gradient hook
(``flashns_v8_coordinate_wgrad``) match the dense contraction bar_Z^T X of the packed
coordinate jets, structural zeros included, as the reference's tests/test_coordinate_wgrad.py:55-70
requires of its own kernel: a non-finite value in a higher-order slot contaminates dW
through 0 * NaN but never db, and a unit slot keeps its matching Inf."""

import math

import pytest
import torch

from tests.cases import close_ratio

pytestmark = pytest.mark.gpu


def dense_contraction(layout, x, d):
    """(bar_Z^T X, sum of bar_Z over order-0 rows) as elementwise IEEE products, so no
    library GEMM can skip a zero."""
    coords = layout.coordinates(x)
    dw = (d[:, :, None] * coords[:, None, :]).sum(0)
    return dw, d[layout.zero_rows(x.device)].sum(0)


def assert_patterns(actual, expected):
    for got, want in zip(actual, expected):
        got = got.cpu()
        for predicate in (torch.isnan, torch.isposinf, torch.isneginf):
            assert torch.equal(predicate(got), predicate(want))
        finite = torch.isfinite(want)
        assert close_ratio(got[finite].numpy(), want[finite].numpy()) <= 1


@pytest.mark.parametrize("dim", [2, 3])
def test_each_nonfinite_slot_propagates_like_the_dense_contraction(cuda, dim):
    from flashns_b200.jet_packed import PackedLayout
    from flashns_b200.native import NativeCUDA
    nat = NativeCUDA()
    layout = PackedLayout(1, 1, dim)
    x = torch.ones(layout.points, dim, dtype=torch.float64)
    for slot in range(layout.rows):
        for value in (math.nan, math.inf, -math.inf):
            d = torch.zeros(layout.rows, 3, dtype=torch.float64)
            d[slot, 1] = value
            got = nat.coordinate_wgrad(layout, x.to(cuda), d.to(cuda))
            assert_patterns(got, dense_contraction(layout, x, d))
    # +Inf on the unit slot of axis 0: dW[0, 0] = +Inf, the other axes NaN, db untouched
    d = torch.zeros(layout.rows, 1, dtype=torch.float64)
    d[dim, 0] = math.inf
    dw, db = nat.coordinate_wgrad(layout, x.to(cuda), d.to(cuda))
    dw, db = dw.cpu(), db.cpu()
    assert torch.isposinf(dw[0, 0]) and bool(torch.isnan(dw[0, 1:]).all())
    assert db.item() == 0.0


@pytest.mark.parametrize("dim", [2, 3])
def test_finite_values_unchanged_by_the_structural_zeros(cuda, dim):
    from flashns_b200.jet_packed import PackedLayout
    from flashns_b200.native import NativeCUDA
    layout = PackedLayout(17, 5, dim)
    gen = torch.Generator(device="cpu").manual_seed(89917)
    x = torch.randn(layout.points, dim, generator=gen, dtype=torch.float64) * 0.3
    d = torch.randn(layout.rows, 7, generator=gen, dtype=torch.float64) * 0.3
    got = NativeCUDA().coordinate_wgrad(layout, x.to(cuda), d.to(cuda))
    for g, e in zip(got, dense_contraction(layout, x, d)):
        assert close_ratio(g.cpu().numpy(), e.numpy()) <= 1

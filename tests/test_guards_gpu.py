"""GPU: guard regions around the caller's output and workspace stay untouched, and
NaN-prefilled outputs and scratch never leak into the results.

compute-sanitizer is not available on the GPU pool, so these checks stand in for its
memcheck and initcheck.  Every evaluation writes through the C ABI into views that
have 8-double sentinel guards on both sides.  The views stay 16-byte aligned.  The
shapes cover every kernel path:

* fused 64-wide layers, with boundary tiles that leave thread-column slots empty;
* value boundary rows;
* the uvp head without boundary points;
* 3-D;
* the 128-wide non-fused path;
* padded widths, which take the packing kernel path.

Segment sizes are ragged.
"""

import ctypes

import numpy as np
import pytest
import torch

from tests.cases import flat, random_case

pytestmark = pytest.mark.gpu

GUARD = 8
SENTINEL = -7.77e307

CASES = [
    ("psi", 1, [2, 64, 64, 64, 2], 333, 97),
    ("psi", 0, [2, 64, 64, 64, 2], 250, 61),
    ("uvp", 0, [2, 64, 64, 3], 177, 0),
    ("psi", 1, [3, 64, 64, 2], 91, 37),
    ("psi", 1, [2, 128, 128, 2], 120, 40),
    ("psi", 1, [2, 40, 72, 2], 60, 21),
]


def guarded(n, device, fill):
    buf = torch.full((n + 2 * GUARD,), SENTINEL, dtype=torch.float64, device=device)
    view = buf[GUARD:GUARD + n]
    view.fill_(fill)
    return buf, view


def guards_intact(buf, n):
    return bool((buf[:GUARD] == SENTINEL).all()) and bool((buf[GUARD + n:] == SENTINEL).all())


@pytest.mark.parametrize("head,order,widths,ni,nb", CASES)
def test_guards_and_nan_prefill(cuda, head, order, widths, ni, nb):
    from flashns_b200 import _lib
    from flashns_b200.evaluator import PackedEvaluator
    from flashns_b200.ns_seed import NSLoss

    case = random_case(ni, nb, widths, head=head, boundary_order=order, seed=ni + nb)
    t = lambda a: torch.tensor(a, dtype=torch.float64)
    loss = NSLoss(0.05, 0.2 if head == "uvp" else 0.0, 3.0)
    ev = PackedEvaluator(t(case["x"]), case["ni"], t(case["pw"]), t(case["bw"]), t(case["target"]), widths,
                         head=head, boundary_order=order, loss=loss, device=cuda)
    params = t(flat(case["ws"], case["bs"])).to(cuda)
    expected = ev(params).cpu().numpy()
    n_out, n_ws = ev.parameters + 1, ev.plan.workspace_bytes // 8
    out_buf, out = guarded(n_out, cuda, float("nan"))
    ws_buf, ws = guarded(n_ws, cuda, float("nan"))  # scratch starts as NaN: nothing may read it unwritten
    ptr = lambda x: ctypes.c_void_p(x.data_ptr()) if x.numel() else None
    stream = torch.cuda.current_stream(cuda)
    for _ in range(2):  # the second call starts from the scratch the first one left
        status = _lib.library().flashns_b200_eval(ev.plan.handle, ptr(ev.x), ptr(params), ptr(ev.pde_weights),
                                                  ptr(ev.boundary_weights), ptr(ev.target), ptr(out), ptr(ws),
                                                  n_ws * 8, ctypes.c_void_p(stream.cuda_stream))
        assert status == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        np.testing.assert_array_equal(got, expected)  # same plan, fixed-order reductions
        assert guards_intact(out_buf, n_out) and guards_intact(ws_buf, n_ws)


@pytest.mark.parametrize("dim,order", [(2, 1), (3, 1), (2, 0)])
def test_field_output_guards(cuda, dim, order):
    from flashns_b200.evaluator import FieldEvaluator, flat_parameters, target_width, xavier_normal

    widths = [dim, 64, 64, 64, 2]
    gen = torch.Generator(device="cpu").manual_seed(dim * 10 + order)
    x = torch.rand(777, dim, generator=gen, dtype=torch.float64)
    fe = FieldEvaluator(x, widths, head="psi", boundary_order=order, device=cuda)
    ws, bs = xavier_normal(widths, 3)
    p = flat_parameters(ws, bs).to(cuda)
    expected = fe(p).cpu().numpy()
    width = target_width("psi", order)
    n = len(x) * width
    buf, view = guarded(n, cuda, float("nan"))
    got = fe(p, view.view(len(x), width))
    torch.cuda.synchronize()
    assert np.isfinite(got.cpu().numpy()).all()
    np.testing.assert_array_equal(got.cpu().numpy(), expected)
    assert guards_intact(buf, n)


def test_field_evaluator_rejects_a_wrong_output_buffer(cuda):
    """A caller-supplied fields buffer of the wrong shape, dtype or layout is refused
    before anything is launched (the kernel writes points x F values)."""
    from flashns_b200.evaluator import FieldEvaluator, flat_parameters, xavier_normal

    widths = [2, 64, 64, 2]
    x = torch.rand(50, 2, generator=torch.Generator(device="cpu").manual_seed(5), dtype=torch.float64)
    fe = FieldEvaluator(x, widths, head="psi", boundary_order=1, device=cuda)
    p = flat_parameters(*xavier_normal(widths, 1)).to(cuda)
    for bad in (torch.empty(49, 3, dtype=torch.float64, device=cuda),
                torch.empty(50, 2, dtype=torch.float64, device=cuda),
                torch.empty(50, 3, dtype=torch.float32, device=cuda),
                torch.empty(3, 50, dtype=torch.float64, device=cuda).T):
        with pytest.raises(ValueError):
            fe(p, bad)

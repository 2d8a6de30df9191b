"""GPU: the no-allocation entry point, through the C ABI.

flashns_b200_eval_static serves callers that cannot allocate device memory (for
example a Go or Java process bound to the C ABI with no CUDA allocator of its own):
it keeps its scratch in a fixed 64 MiB device array inside the library instead of a
caller workspace.  Its output must match flashns_b200_eval on two calls in a row, after
another plan's call has filled the array with unrelated values (every call reuses the
array as the previous one left it).  This file is collected
last so that a run stopping at the first failure has run every other test first.
"""

import ctypes

import numpy as np
import pytest
import torch

from tests.cases import close_ratio, flat, random_case

pytestmark = pytest.mark.gpu


def _evaluator(cuda, widths, ni, nb, seed):
    from flashns_b200.evaluator import PackedEvaluator
    from flashns_b200.ns_seed import NSLoss
    case = random_case(ni, nb, widths, head="psi", boundary_order=1, seed=seed)
    t = lambda a: torch.tensor(a, dtype=torch.float64)
    ev = PackedEvaluator(t(case["x"]), case["ni"], t(case["pw"]), t(case["bw"]), t(case["target"]), widths,
                         head="psi", boundary_order=1, loss=NSLoss(0.05), device=cuda)
    assert ev.plan.workspace_bytes <= 64 * 1024 * 1024
    return ev, t(flat(case["ws"], case["bs"])).to(cuda)


def _static(lib, ev, params, cuda):
    ptr = lambda x: ctypes.c_void_p(x.data_ptr())
    out = torch.full((ev.parameters + 1,), float("nan"), dtype=torch.float64, device=cuda)
    status = lib.flashns_b200_eval_static(ev.plan.handle, ptr(ev.x), ptr(params), ptr(ev.pde_weights),
                                          ptr(ev.boundary_weights), ptr(ev.target), ptr(out),
                                          ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream))
    assert status == 0
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    return got


def test_static_entry_point_matches_workspace_entry_point(cuda):
    """Two calls in a row of one plan match the workspace entry point, after a call of a
    different plan (3-D, 128 wide) has left its own values all over the shared array; a
    last call of that other plan then finds the array as the 2-D plan left it."""
    from flashns_b200 import _lib

    lib = _lib.library()
    ev, params = _evaluator(cuda, [2, 64, 64, 64, 2], 700, 180, 17)
    other, other_params = _evaluator(cuda, [3, 128, 128, 2], 150, 60, 5)
    expected = ev(params).cpu().numpy()
    other_expected = other(other_params).cpu().numpy()
    assert close_ratio(_static(lib, other, other_params, cuda), other_expected) <= 1.0  # the array is dirty now
    for _ in range(2):
        assert close_ratio(_static(lib, ev, params, cuda), expected) <= 1.0
    assert close_ratio(_static(lib, other, other_params, cuda), other_expected) <= 1.0


def test_static_entry_point_rejects_oversize_plans(cuda):
    from flashns_b200 import _lib
    from flashns_b200.evaluator import PackedEvaluator
    from flashns_b200.ns_seed import NSLoss

    lib = _lib.library()
    widths = [2, 64, 64, 64, 2]
    case = random_case(16384, 64, widths, head="psi", boundary_order=1, seed=3)
    t = lambda a: torch.tensor(a, dtype=torch.float64)
    ev = PackedEvaluator(t(case["x"]), case["ni"], t(case["pw"]), t(case["bw"]), t(case["target"]), widths,
                         head="psi", boundary_order=1, loss=NSLoss(0.05), device=cuda)
    assert ev.plan.workspace_bytes > 64 * 1024 * 1024
    out = torch.zeros(ev.parameters + 1, dtype=torch.float64, device=cuda)
    params = t(flat(case["ws"], case["bs"])).to(cuda)
    ptr = lambda x: ctypes.c_void_p(x.data_ptr())
    status = lib.flashns_b200_eval_static(ev.plan.handle, ptr(ev.x), ptr(params), ptr(ev.pde_weights),
                                          ptr(ev.boundary_weights), ptr(ev.target), ptr(out),
                                          ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream))
    assert status == 1  # cudaErrorInvalidValue: beyond the static capacity, nothing launched
    torch.cuda.synchronize()
    assert bool((out == 0).all())

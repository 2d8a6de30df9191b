"""CPU: the C-ABI library builds, loads and exports every entry point the headers declare."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared():
    names = []
    for header in sorted((ROOT / "include").glob("*.h")):
        names += re.findall(r"^(?:int|void)\s+(\w+)\s*\(", header.read_text(), flags=re.M)
    return names


@pytest.fixture(scope="module")
def library():
    from flashns_b200 import build
    path = build.build()
    return ctypes.CDLL(str(path))


def test_headers_declare_entry_points():
    names = declared()
    assert "flashns_b200_eval" in names and "flashns_b200_plan_create" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol(library):
    missing = [n for n in declared() if not hasattr(library, n)]
    assert not missing, missing


def test_python_binding_covers_declared_symbols(library):
    from flashns_b200 import _lib
    assert set(_lib.SIGNATURES) <= set(declared())
    lib = _lib.library()
    for name in _lib.SIGNATURES:
        assert getattr(lib, name).restype is ctypes.c_int


def test_plan_rejects_invalid_arguments_without_a_gpu(library):
    """Argument checks run before any device query, so they work on a CPU host."""
    from flashns_b200 import _lib
    lib = _lib.library()
    handle = ctypes.c_void_p()
    bad = [
        (4, 1, 1, [4, 64, 2]),     # dim 4
        (2, 0, 1, [2, 64, 3]),     # uvp head with first-order boundary rows
        (3, 0, 0, [3, 64, 3]),     # uvp head in 3-D
        (2, 1, 0, [2, 64, 3]),     # psi head needs 2 outputs
        (2, 1, 0, [2, 2]),         # no hidden layer
        (2, 1, 0, [3, 64, 2]),     # input width != dim
    ]
    for dim, head, order, widths in bad:
        arr = (ctypes.c_int * len(widths))(*widths)
        status = lib.flashns_b200_plan_create(dim, head, order, len(widths) - 1, arr, 10, 5, 0.05, 0.2, 5.0,
                                              ctypes.byref(handle))
        assert status == 1, (dim, head, order, widths, status)  # cudaErrorInvalidValue
        assert not handle.value
    # more packed rows than 32-bit tile coordinates address: 2^28 2-D interior points are
    # 2.7e9 rows; (2^31 - 1) / 10 points with one value point is one row too many
    arr = (ctypes.c_int * 3)(2, 64, 2)
    for ni, nb in ((1 << 28, 0), ((2**31 - 1) // 10, 8), (0, 2**31)):
        status = lib.flashns_b200_plan_create(2, 1, 0, 2, arr, ni, nb, 0.05, 0.2, 5.0, ctypes.byref(handle))
        assert status == 1 and not handle.value, (ni, nb)


def test_no_fallback_when_library_missing(tmp_path, monkeypatch):
    from flashns_b200 import _lib
    monkeypatch.setattr(_lib, "LIBRARY", tmp_path / "absent.so")
    monkeypatch.setattr(_lib, "_library", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.library()


def test_hopper_plan_names_reject_bad_arguments(library):
    """The reference's Hopper plan limits (experiments/cuda_jet_hopper/hopper.cu:303-310),
    checked on the host before any CUDA call."""
    from flashns_b200 import _lib
    lib = _lib.library()
    plan = ctypes.c_void_p()
    p16, p8 = ctypes.c_void_p(16), ctypes.c_void_p(24)
    assert lib.flashns_hopper_create(2, p16, p16, 10, 48, 64, ctypes.byref(plan)) == 1   # cout not 32/64
    assert lib.flashns_hopper_create(2, p16, p16, 10, 64, 16, ctypes.byref(plan)) == 1   # cin not 32/64
    assert lib.flashns_hopper_create(4, p16, p16, 10, 64, 64, ctypes.byref(plan)) == 1   # dim
    assert lib.flashns_hopper_create(2, p16, p16, 0, 64, 64, ctypes.byref(plan)) == 1    # empty batch
    assert lib.flashns_hopper_create(2, p8, p16, 10, 64, 64, ctypes.byref(plan)) == 1    # D not 16-byte aligned
    assert lib.flashns_hopper_create(2, None, p16, 10, 64, 64, ctypes.byref(plan)) == 1
    assert lib.flashns_hopper_create(2, p16, p16, 10, 64, 64, None) == 1
    assert lib.flashns_hopper_create(3, p16, p16, 10, 32, 64, ctypes.byref(plan)) == 0 and plan.value
    try:
        assert lib.flashns_hopper_launch(plan, 2, False, None, None, p16, None) == 1      # plan is 3-D
        assert lib.flashns_hopper_launch(plan, 3, True, None, None, p16, None) == 1       # fused needs H, a1
        assert lib.flashns_hopper_launch(plan, 3, False, None, None, None, None) == 1     # no output
        assert lib.flashns_hopper_launch(None, 3, False, None, None, p16, None) == 1
    finally:
        lib.flashns_hopper_destroy(plan)


def test_hook_entry_points_check_arguments_before_any_launch(library):
    """The reference's hook ABI (experiments/pinn_v8/native.cu:47-62,97-107,
    experiments/cuda_jet_h100/stable_kernels.cu:82-131, stable_dgrad.cu:150-174): invalid
    sizes and missing or aliased buffers return cudaErrorInvalidValue (1), and empty inputs
    return success, before anything is launched -- so this runs on a CPU host.  The
    pointers are never dereferenced."""
    from flashns_b200 import _lib
    lib = _lib.library()
    p, q, r = ctypes.c_void_p(4096), ctypes.c_void_p(1 << 20), ctypes.c_void_p(1 << 24)
    big = 1 << 62
    act = lib.flashns_v8_activation
    assert act(4, 0, p, None, None, q, r, 3, 2, 8, None) == 1           # dimension
    assert act(2, 2, p, None, None, q, r, 3, 2, 8, None) == 1           # backward flag
    assert act(2, 0, p, None, None, q, r, -1, 2, 8, None) == 1          # negative points
    assert act(2, 0, p, None, None, q, r, 3, 2, 0, None) == 1           # no channels
    assert act(2, 0, p, None, None, q, r, big, 0, 8, None) == 1         # rows overflow
    assert act(2, 0, None, None, None, q, r, 3, 2, 8, None) == 1        # no input
    assert act(2, 1, p, None, p, q, None, 3, 2, 8, None) == 1           # VJP without a1
    assert act(3, 1, None, None, None, None, None, 0, 0, 8, None) == 0  # empty: success
    for fn in (lib.flashns_v8_coordinate_affine,):
        assert fn(2, p, q, r, p, 3, 2, 0, None) == 1
        assert fn(2, p, q, None, p, 3, 2, 8, None) == 1                 # no bias
        assert fn(2, None, None, None, None, 0, 0, 8, None) == 0
    assert lib.flashns_v8_coordinate_affine_activation(2, p, q, r, p, None, 3, 2, 8, None) == 1  # no a1 out
    tail = lib.flashns_v8_tail3
    assert tail(2, 2, p, q, r, p, q, 3, 2, 8, None) == 1                # fused flag
    assert tail(2, 1, p, q, None, p, q, 3, 2, 8, None) == 1             # fused without H
    assert tail(2, 0, None, None, None, None, None, 0, 0, 8, None) == 0
    wg = lib.flashns_v8_coordinate_wgrad
    assert wg(2, p, q, r, None, p, 3, 2, 8, None) == 1                  # no dW
    assert wg(2, p, None, r, q, p, 3, 2, 8, None) == 1                  # no coordinates
    assert wg(5, p, q, r, q, p, 3, 2, 8, None) == 1
    assert lib.flashns_v8_coordinate_activation_wgrad(2, p, None, p, q, r, q, p, 3, 2, 8, None) == 1  # no a1
    seed = lib.flashns_v8_loss_seed
    assert seed(p, p, p, p, p, q, q, r, 4, 2, 2, 0.07, 0.2, 5.0, None) == 1   # boundary stride < 3
    assert seed(p, p, p, p, p, q, q, r, -1, 2, 3, 0.07, 0.2, 5.0, None) == 1
    assert seed(p, p, p, p, p, q, q, None, 4, 2, 3, 0.07, 0.2, 5.0, None) == 1  # no loss partials
    assert seed(p, None, p, p, p, q, q, r, 4, 2, 3, 0.07, 0.2, 5.0, None) == 1  # boundary missing
    assert seed(None, None, None, None, None, None, None, None, 0, 0, 3, 0.07, 0.2, 5.0, None) == 0
    sa = lib.flashns_stable_activation
    assert sa(1, False, p, None, None, q, r, 4, 8, None) == 1
    assert sa(2, False, p, None, None, p, r, 4, 8, None) == 1           # output aliases input
    assert sa(2, True, p, q, r, p, None, 4, 8, None) == 1               # output aliases H
    assert sa(2, False, p, None, None, q, None, 4, 8, None) == 1        # no a1 out
    assert sa(3, False, None, None, None, None, None, 0, 8, None) == 0
    dg = lib.flashns_stable_dgrad_vjp
    assert dg(2, False, p, q, None, None, r, -1, 8, 8, None) == 1
    assert dg(2, False, p, q, None, None, r, 4, 0, 8, None) == 1        # cout 0
    assert dg(2, True, p, q, None, None, r, 4, 8, 8, None) == 1         # fused without H, a1
    assert dg(2, False, p, q, None, None, p, 4, 8, 8, None) == 1        # output aliases D
    assert dg(2, False, None, None, None, None, None, 0, 8, 8, None) == 0


def test_fp64_probe_rejects_bad_launch_shapes(library):
    """The peak-table probe checks its kind and launch shape before launching."""
    from flashns_b200 import _lib
    from baseline.fp64_peak import KINDS
    lib = _lib.library()
    sink, flops = ctypes.c_void_p(4096), ctypes.c_double()
    probe = lambda kind, blocks, threads, iters, s=sink: lib.flashns_b200_fp64_probe(kind, blocks, threads, iters, s,
                                                                                      ctypes.byref(flops), None)
    assert sorted(KINDS.values()) == list(range(6))
    assert probe(6, 148, 256, 10) == 1 and probe(-1, 148, 256, 10) == 1
    assert probe(1, 148, 100, 10) == 1 and probe(1, 148, 2048, 10) == 1     # threads
    assert probe(0, 148, 512, 10) == 1                                      # m16n8k8 runs at 256 threads
    assert probe(2, 0, 256, 10) == 1 and probe(2, 148, 256, 0) == 1
    assert probe(5, 148, 256, 10, None) == 1

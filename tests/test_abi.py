"""CPU: the C-ABI library builds, loads and exports every entry point the headers declare."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared():
    names = []
    for header in sorted((ROOT / "include").glob("*.h")):
        names += re.findall(r"^int\s+(\w+)\s*\(", header.read_text(), flags=re.M)
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


def test_no_fallback_when_library_missing(tmp_path, monkeypatch):
    from flashns_b200 import _lib
    monkeypatch.setattr(_lib, "LIBRARY", tmp_path / "absent.so")
    monkeypatch.setattr(_lib, "_library", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.library()

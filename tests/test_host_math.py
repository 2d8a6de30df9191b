"""CPU: the product's generated device arithmetic, compiled as host C++, against the
oracle.

``tests/host_math.cpp`` includes ``flashns_b200/csrc/jets_generated.cuh`` and
``residual_generated.cuh`` -- the stable-tanh jets, their VJPs and the residual seeds that
every evaluation kernel inlines -- and g++ builds them with ``-ffp-contract=off`` (the
reference compiles its shared ``.cuh`` math the same way,
``experiments/pinn_v8/coordinate_wgrad_host.py``).  The formulas are checked on every
order and dimension the kernels use, saturated centers included, without a GPU.
"""

import ctypes
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import jets as J
from oracle import residuals as RS
from tests.cases import close_ratio

ROOT = Path(__file__).resolve().parents[1]
D = ctypes.POINTER(ctypes.c_double)


@pytest.fixture(scope="module")
def host(tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    out = tmp_path_factory.mktemp("host_math") / "host_math.so"
    subprocess.run([gxx, "-O2", "-std=c++17", "-ffp-contract=off", "-shared", "-fPIC",
                    f"-I{ROOT / 'flashns_b200' / 'csrc'}", str(ROOT / "tests" / "host_math.cpp"), "-o", str(out)],
                   check=True, capture_output=True)
    lib = ctypes.CDLL(str(out))
    lib.host_jet_fwd.argtypes = [ctypes.c_int, ctypes.c_int, D, D, D, ctypes.c_long]
    lib.host_jet_vjp.argtypes = [ctypes.c_int, ctypes.c_int, D, D, D, D, ctypes.c_long]
    lib.host_seed.argtypes = [ctypes.c_int, ctypes.c_int, D, D, ctypes.c_double, ctypes.c_double, D, D, ctypes.c_long]
    lib.host_residuals.argtypes = [ctypes.c_int, ctypes.c_int, D, ctypes.c_double, D, ctypes.c_long]
    return lib


def ptr(a):
    return a.ctypes.data_as(D)


def jets(rng, n, dim, order):
    q = len(J.basis(dim, order))
    z = rng.normal(size=(n, q)) * 0.4
    z[:4, 0] = (20.0, -20.0, 350.0, 1e-4)  # saturated both ways, far tail, the small-|z| series
    return z


@pytest.mark.parametrize("dim", [2, 3])
@pytest.mark.parametrize("order", [0, 1, 3])
def test_generated_jet_and_vjp_match_oracle(host, dim, order):
    rng = np.random.default_rng(100 * dim + order)
    z = jets(rng, 37, dim, order)
    h, a1 = np.zeros_like(z), np.zeros(len(z))
    assert host.host_jet_fwd(dim, order, ptr(z), ptr(h), ptr(a1), len(z)) == 0
    hr, ar = J.tanh_jet(z[:, :, None], dim, order)
    assert close_ratio(h, hr[:, :, 0]) <= 1 and close_ratio(a1, ar[:, 0]) <= 1
    hb = rng.normal(size=z.shape)
    zb = np.zeros_like(z)
    assert host.host_jet_vjp(dim, order, ptr(h), ptr(a1), ptr(hb), ptr(zb), len(z)) == 0
    assert close_ratio(zb, J.tanh_vjp(hr, ar, hb[:, :, None], dim, order)[:, :, 0]) <= 1


@pytest.mark.parametrize("head,dim,outputs", [(0, 2, 3), (1, 2, 2), (1, 3, 2)])
@pytest.mark.parametrize("nu,gamma", [(0.07, 0.2), (0.01, 0.0), (0.05, 1.3)])
def test_generated_seed_and_residuals_match_oracle(host, head, dim, outputs, nu, gamma):
    rng = np.random.default_rng(7 + head + dim)
    y = rng.normal(size=(29, J.q(dim), outputs)) * 0.4
    w = rng.uniform(0.0, 1.0, size=29)
    w[0] = 0.0
    dy, loss = np.zeros_like(y), np.zeros(29)
    assert host.host_seed(head, dim, ptr(y), ptr(w), nu, gamma, ptr(dy), ptr(loss), 29) == 0
    name = "uvp" if head == 0 else "psi"
    ref_loss, ref_seed = RS.interior_seed(y, w, name, nu, gamma)
    assert close_ratio(loss, ref_loss) <= 1 and close_ratio(dy, ref_seed) <= 1
    ref_r = RS.residual_values(y, name, nu, gamma)
    r = np.zeros_like(ref_r)
    assert host.host_residuals(head, dim, ptr(y), nu, ptr(r), 29) == 0
    assert close_ratio(r, ref_r) <= 1


def test_unsupported_shapes_are_refused(host):
    z = np.zeros((1, 20))
    assert host.host_jet_fwd(2, 2, ptr(z), ptr(z.copy()), ptr(np.zeros(1)), 1) == 1
    assert host.host_seed(0, 3, ptr(z), ptr(np.zeros(1)), 0.1, 0.2, ptr(z.copy()), ptr(np.zeros(1)), 1) == 1

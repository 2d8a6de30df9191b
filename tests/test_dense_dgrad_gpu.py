"""GPU: the dense dgrad (+ jet VJP) behind the reference's fused-dgrad ABI
(``flashns_stable_dgrad_vjp``, experiments/cuda_jet_h100/stable_dgrad.cu:150-174), a DMMA
mainloop with the VJP in its epilogue, against the oracle.

Shapes cover K (cout) and channel (cin) sizes that are not multiples of the 32-wide K
chunk or the 64-wide channel block, a single sample, sample counts that leave a partial
tile, and the reference's published local shape (B = 16,384, 64 -> 64).  Every output
element must be written (NaN prefill) and nothing outside the output (sentinel guards);
values within the reference criterion ``|a-b| <= 2e-12 + 2e-11|b|``.
"""

import ctypes

import numpy as np
import pytest
import torch

from tests.cases import close_ratio

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1, 1), (9, 3, 13), (37, 64, 64), (300, 37, 70), (129, 128, 100), (77, 5, 129)]


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _run(lib, cuda, dim, fused, d, w, h, a1, guard=64):
    from oracle import jets as J
    batch, q, cout = d.shape
    cin = w.shape[1]
    T = lambda a: torch.tensor(np.ascontiguousarray(a), dtype=torch.float64, device=cuda)
    dg, wg = T(d), T(w)
    hg, ag = (T(h), T(a1)) if fused else (None, None)
    n = batch * q * cin
    buf = torch.full((n + 2 * guard,), float("nan"), dtype=torch.float64, device=cuda)
    buf[:guard] = 7.0
    buf[guard + n:] = -7.0
    out = buf[guard:guard + n]
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    assert lib.flashns_stable_dgrad_vjp(dim, fused, _ptr(dg), _ptr(wg), _ptr(hg), _ptr(ag), _ptr(out), batch, cout,
                                        cin, stream) == 0
    torch.cuda.synchronize()
    host = buf.cpu().numpy()
    assert (host[:guard] == 7.0).all() and (host[guard + n:] == -7.0).all(), "write outside the output"
    got = host[guard:guard + n].reshape(batch, q, cin)
    assert np.isfinite(got).all(), "output element not written"
    dh = d @ w
    return got, (J.tanh_vjp(h, a1, dh, dim) if fused else dh)


@pytest.mark.parametrize("dim", [2, 3])
@pytest.mark.parametrize("batch,cout,cin", SHAPES)
def test_dense_dgrad_matches_oracle(cuda, dim, batch, cout, cin):
    from flashns_b200 import _lib
    from oracle import jets as J
    lib = _lib.library()
    rng = np.random.default_rng(batch * 1000 + cout * 10 + cin)
    q = J.q(dim)
    z = rng.normal(size=(batch, q, cin)) * 0.5
    z[0, 0, :] += 15.0  # a saturated sample
    h, a1 = J.tanh_jet(z, dim)
    d = rng.normal(size=(batch, q, cout))
    w = rng.normal(size=(cout, cin)) / np.sqrt(cout)
    for fused in (False, True):
        got, expect = _run(lib, cuda, dim, fused, d, w, h, a1)
        assert close_ratio(got, expect) <= 1.0, (dim, batch, cout, cin, fused)


def test_dense_dgrad_at_the_reference_local_shape(cuda):
    """B = 16,384 samples, 64 -> 64, 2-D (the shape of the reference's local dgrad + VJP
    timing, docs/cuda-h100-results.md:112-120): many tiles per CTA of the persistent grid."""
    from flashns_b200 import _lib
    from oracle import jets as J
    lib = _lib.library()
    rng = np.random.default_rng(16384)
    z = rng.normal(size=(16384, 10, 64)) * 0.5
    h, a1 = J.tanh_jet(z, 2)
    d = rng.normal(size=(16384, 10, 64)) / 16384
    w = rng.normal(size=(64, 64)) / 8.0
    got, expect = _run(lib, cuda, 2, True, d, w, h, a1)
    assert close_ratio(got, expect) <= 1.0


def test_dense_dgrad_rejects_bad_arguments(cuda):
    from flashns_b200 import _lib
    lib = _lib.library()
    x = torch.zeros(64, dtype=torch.float64, device=cuda)
    p = _ptr(x)
    assert lib.flashns_stable_dgrad_vjp(4, False, p, p, None, None, _ptr(x[32:]), 1, 1, 1, None) == 1
    assert lib.flashns_stable_dgrad_vjp(2, True, p, p, None, None, _ptr(x[32:]), 1, 1, 1, None) == 1
    assert lib.flashns_stable_dgrad_vjp(2, False, p, p, None, None, None, 0, 1, 1, None) == 0  # empty
    assert lib.flashns_stable_dgrad_shared_bytes() > 0


@pytest.mark.parametrize("dim", [2, 3])
def test_dense_dgrad_with_h_and_a1_views_off_a_16_byte_boundary(cuda, dim):
    """64 -> 64 with H and a1 passed as views one double into larger buffers (8-byte but not
    16-byte aligned): the hook takes the general kernel instead of the fused kernels, whose
    bulk L2 prefetches want 16-byte aligned rows, and the values still match the oracle."""
    from flashns_b200 import _lib
    from oracle import jets as J
    lib = _lib.library()
    rng = np.random.default_rng(4242 + dim)
    q, batch = J.q(dim), 129
    z = rng.normal(size=(batch, q, 64)) * 0.5
    h, a1 = J.tanh_jet(z, dim)
    d = rng.normal(size=(batch, q, 64))
    w = rng.normal(size=(64, 64)) / 8.0
    T = lambda a: torch.tensor(np.ascontiguousarray(a), dtype=torch.float64, device=cuda)
    hbuf = torch.zeros(h.size + 1, dtype=torch.float64, device=cuda)
    abuf = torch.zeros(a1.size + 1, dtype=torch.float64, device=cuda)
    hbuf[1:] = T(h).reshape(-1)
    abuf[1:] = T(a1).reshape(-1)
    hv, av = hbuf[1:], abuf[1:]
    assert hv.data_ptr() % 16 == 8 and av.data_ptr() % 16 == 8
    dg, wg = T(d), T(w)
    out = torch.full((batch * q * 64,), float("nan"), dtype=torch.float64, device=cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    assert lib.flashns_stable_dgrad_vjp(dim, True, _ptr(dg), _ptr(wg), _ptr(hv), _ptr(av), _ptr(out), batch, 64, 64,
                                        stream) == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy().reshape(batch, q, 64)
    assert np.isfinite(got).all()
    assert close_ratio(got, J.tanh_vjp(h, a1, d @ w, dim)) <= 1.0
